"""Generate the committed golden fixtures under tests/golden/.

Run where the reference tree is present (its path as the first argument, else
MLXTURBO_REFERENCE_ROOT, else a `reference` directory beside this repository):

    python tests/golden/make_golden.py [REFERENCE_ROOT]

Fixtures (all small, all seeded):

  dequant_ref.npz  packed rows for bits 2,3,4,5,6,8 and their dequantised
                   values computed by the reference's own `dequantize` template
                   (compiled by oracle/ref_dequant/build_ref.py), as fp32
                   (U=float) and as bf16 (U=bfloat).
  pack_ref.npz     codes and the uint32 words produced by the reference's numpy
                   packer `quantize_affine` (tools/ane_quant_probe.py:34-50) for
                   bits 4 and 8 -- pins the low-bits-first word layout.
  route_table.json routes from the reference's pure-Python router
                   (mlxturbo/kernels/dispatch.py:102-117, 247-299) for every
                   table key, M = -1..20, and the small-M override rows.

The tests read only these files; nothing at test time touches the reference.
"""

from __future__ import annotations

import ast
import importlib.util
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle", "ref_dequant"))


def bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def make_dequant(ref_root: str) -> None:
    import build_ref

    exe = build_ref.build(ref_root)
    rng = np.random.default_rng(1234)
    K, rows = 128, 48
    out = {}
    for bits in (2, 3, 4, 5, 6, 8):
        nbytes = K * bits // 8
        packed = rng.integers(0, 256, size=(rows, nbytes), dtype=np.uint8)
        packed[0, :] = 0
        packed[1, :] = 255
        s = rng.normal(0, 0.02, size=rows).astype(np.float32)
        b = rng.normal(0, 0.05, size=rows).astype(np.float32)
        s[2], b[2] = -0.03125, 0.0          # negative scale (MLX max-edge groups)
        s[3], b[3] = 1.0e-7, -1.5           # degenerate group
        s[4], b[4] = 3.0, 100.0             # large magnitudes
        sh, bh = bf16_round(s), bf16_round(b)
        s32, b32 = bf16_to_f32(sh), bf16_to_f32(bh)
        payload = np.array([bits, rows, K], dtype=np.int32).tobytes()
        for r in range(rows):
            payload += s32[r:r + 1].tobytes() + b32[r:r + 1].tobytes() + packed[r].tobytes()
        res = subprocess.run([exe], input=payload, capture_output=True, check=True).stdout
        rec = np.frombuffer(res, dtype=np.uint8).reshape(rows, K * 4 + K * 2)
        deq_f32 = rec[:, :K * 4].copy().view(np.float32)
        deq_bf16 = rec[:, K * 4:].copy().view(np.uint16)
        out[f"b{bits}_words"] = packed.view(np.uint32).reshape(rows, K * bits // 32)
        out[f"b{bits}_scales"] = sh.reshape(rows, 1)
        out[f"b{bits}_biases"] = bh.reshape(rows, 1)
        out[f"b{bits}_deq_f32"] = deq_f32
        out[f"b{bits}_deq_bf16"] = deq_bf16
    np.savez_compressed(os.path.join(HERE, "dequant_ref.npz"), K=K, **out)


def _load_function(path: str, name: str):
    tree = ast.parse(open(path, encoding="utf-8").read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == name)
    mod = ast.Module(body=[fn], type_ignores=[])
    ns = {"np": np}
    exec(compile(mod, path, "exec"), ns)  # noqa: S102 - the reference's own pure-numpy helper
    return ns[name]


def make_pack(ref_root: str) -> None:
    quantize_affine = _load_function(os.path.join(ref_root, "tools", "ane_quant_probe.py"), "quantize_affine")
    rng = np.random.default_rng(99)
    out = {}
    for bits in (4, 8):
        w = rng.normal(0, 0.02, size=(16, 256)).astype(np.float32)
        packed, mn, scale = quantize_affine(w, 64, bits)
        g = w.reshape(16, -1, 64)
        codes = np.round((g - mn[..., None]) / scale[..., None]).astype(np.uint32).reshape(16, 256)
        out[f"b{bits}_codes"] = codes.astype(np.uint8)
        out[f"b{bits}_words"] = packed.astype(np.uint32)
    np.savez_compressed(os.path.join(HERE, "pack_ref.npz"), **out)


def make_routes(ref_root: str) -> None:
    path = os.path.join(ref_root, "mlxturbo", "kernels", "dispatch.py")
    spec = importlib.util.spec_from_file_location("_ref_dispatch", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    table = {f"{k},{n}": list(row) for (k, n), row in mod.DEFAULT_ROUTE_TABLE.items()}
    select = {}
    for (k, n) in list(mod.DEFAULT_ROUTE_TABLE) + [(4096, 11008), (2560, 640)]:
        select[f"{k},{n}"] = [mod.select_route(k, n, m) for m in range(-1, 21)]
    small = {}
    shapes = list(mod.DEFAULT_ROUTE_TABLE) + [(4096, 11008), (5120, 6144), (6144, 5120), (1024, 1024),
                                               (5120, 48), (512, 4096)]
    for route in ("small_m", "nocap", "mma", "off"):
        os.environ["MLXTURBO_SMALL_M_ROUTE"] = route
        mod.refresh_small_m_route()
        small[route] = {f"{k},{n}": (None if (r := mod._small_m_row(k, n)) is None else list(r))
                        for (k, n) in shapes} if route != "off" else {}
    os.environ.pop("MLXTURBO_SMALL_M_ROUTE", None)
    doc = {
        "source": "mlxturbo/kernels/dispatch.py (select_route :102-117, _small_m_row :279-299)",
        "table": table,
        "select_route_m_-1_to_20": select,
        "small_m_rows": small,
        "small_m_window": [mod._SMALL_M_MIN, mod._SMALL_M_MAX],
        "small_m_min_nk": [mod._SMALL_M_N_MIN, mod._SMALL_M_K_MIN],
        "mma_m_min": mod._MMA_M_MIN,
    }
    with open(os.path.join(HERE, "route_table.json"), "w") as f:
        json.dump(doc, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    root = (sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MLXTURBO_REFERENCE_ROOT")
            or os.path.join(os.path.dirname(repo), "reference"))
    make_dequant(root)
    make_pack(root)
    make_routes(root)
    print("golden fixtures written to", HERE)
