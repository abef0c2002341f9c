"""Build oracle/_ref/dequant_ref from the reference's own dequantisation code.

TEST INFRASTRUCTURE ONLY.  The reference ships MLX's `dequantize` template
(quantized.h:483-569) and the pack-factor helpers (quantized.h:12-26) as text
inside mlxturbo/kernels/_steel_flat.py.  This script reads that file from the
reference tree at build time, cuts out exactly those two blocks (between their
"// ---- quantized.h:..." markers), compiles them as C++ with empty Metal
address-space qualifiers, and links a small driver that dequantises packed rows
read from stdin.  Nothing is copied into this repository: the extracted source
and the binary are written under oracle/_ref/ only (git-ignored).

The binary is used by tests/golden/make_golden.py to produce the committed
golden vectors tests/golden/dequant_ref.npz, which pin the oracle's code
unpacking and s*q+b arithmetic bit for bit.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(os.path.dirname(HERE), "_ref")
# the reference checkout: MLXTURBO_REFERENCE_ROOT, else a `reference` directory beside this repository
DEFAULT_REF = os.environ.get("MLXTURBO_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))), "reference")
STEEL = os.path.join("mlxturbo", "kernels", "_steel_flat.py")

BLOCKS = (
    "// ---- quantized.h:12-26 (get_pack_factor / get_bytes_per_pack) ----",
    "// ---- quantized.h:483-569 (dequantize) ----",
)

PRELUDE = r"""
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <vector>
#define device
#define threadgroup
#define thread
#define constant
/* bf16 storage type with Metal's float -> bfloat conversion (round to nearest even). */
struct bf16_t {
  uint16_t bits;
  bf16_t() : bits(0) {}
  bf16_t(float f) {
    uint32_t u; std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) { bits = (uint16_t)((u >> 16) | 0x40u); return; }
    u += 0x7fffu + ((u >> 16) & 1u);
    bits = (uint16_t)(u >> 16);
  }
  operator float() const { uint32_t u = (uint32_t)bits << 16; float f; std::memcpy(&f, &u, 4); return f; }
};
"""

DRIVER = r"""
/* stdin: int32 bits, int32 n_rows, int32 K; then per row: scale(f32) bias(f32)
 * and K*bits/8 bytes.  stdout: per row K float (U=float) then K uint16 (U=bf16). */
template <int bits>
static void run(int rows, int K) {
  constexpr int pf = get_pack_factor<bits>();
  constexpr int bpp = get_bytes_per_pack<bits>();
  std::vector<uint8_t> buf(K * bits / 8);
  std::vector<float> outf(K);
  std::vector<bf16_t> outh(K);
  for (int r = 0; r < rows; ++r) {
    float s, b;
    if (fread(&s, 4, 1, stdin) != 1 || fread(&b, 4, 1, stdin) != 1) exit(2);
    if (fread(buf.data(), 1, buf.size(), stdin) != buf.size()) exit(2);
    for (int p = 0; p < K / pf; ++p) {
      dequantize<float, pf, bits>(buf.data() + p * bpp, s, b, outf.data() + p * pf);
      dequantize<bf16_t, pf, bits>(buf.data() + p * bpp, bf16_t(s), bf16_t(b), outh.data() + p * pf);
    }
    fwrite(outf.data(), 4, K, stdout);
    fwrite(outh.data(), 2, K, stdout);
  }
}
int main() {
  int hdr[3];
  if (fread(hdr, 4, 3, stdin) != 3) return 2;
  switch (hdr[0]) {
    case 2: run<2>(hdr[1], hdr[2]); break;
    case 3: run<3>(hdr[1], hdr[2]); break;
    case 4: run<4>(hdr[1], hdr[2]); break;
    case 5: run<5>(hdr[1], hdr[2]); break;
    case 6: run<6>(hdr[1], hdr[2]); break;
    case 8: run<8>(hdr[1], hdr[2]); break;
    default: return 3;
  }
  return 0;
}
"""


def extract(ref_root: str) -> str:
    text = open(os.path.join(ref_root, STEEL), encoding="utf-8").read()
    parts = []
    for marker in BLOCKS:
        start = text.index(marker)
        end = text.index("// ----", start + len(marker))
        parts.append(text[start:end])
    src = "\n".join(parts)
    # Metal-only spellings used by the two blocks.
    src = src.replace("MLX_MTL_CONST", "static constexpr const")
    src = src.replace("#define static constexpr const static constant constexpr const", "")
    return src


def build(ref_root: str = DEFAULT_REF) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    cpp = os.path.join(OUT_DIR, "dequant_ref.cpp")
    exe = os.path.join(OUT_DIR, "dequant_ref")
    with open(cpp, "w", encoding="utf-8") as f:
        f.write(PRELUDE + extract(ref_root) + DRIVER)
    subprocess.run(["/usr/bin/g++", "-O1", "-std=c++17", "-ffp-contract=off", "-w", "-o", exe, cpp], check=True)
    return exe


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF))
