"""Shared helpers for the parity tests: seeded inputs and the tolerance check.

Tolerance (stated once, used by every matmul parity test), against the fp32
dequantise-then-matmul oracle:
  * normalised max error  max|d| / max(max|ref|, 1)  <= 1e-2
    (the reference's own metric, bench/test_dispatch.py:66-73);
  * mean absolute error   <= MAE of the oracle rounded to the output dtype
                             + 1e-3 * max(1, mean|ref|)
    i.e. at most 1e-3 (relative to output scale) beyond the error that storing
    the exact result in bf16/fp16 already costs.  At the reference tests' input
    scale (x ~ N(0,1)*0.1) this is the plain MAE <= 1e-3 bound.
"""

from __future__ import annotations

import numpy as np
import torch

import oracle as O

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def half_to_torch(h: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(h).view(np.int16)).view(TORCH_DT[dtype]).to(device)


def torch_to_half(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u32_to_torch(w: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(w).view(np.int32)).to(device)


def make_weights(rng, N, K, group_size=64, bits=4, dtype="bf16", std=0.02):
    """Weights ~ N(0, std) through the MLX affine quantiser (oracle)."""
    wf = rng.normal(0, std, size=(N, K)).astype(np.float32)
    return O.quantize(wf, group_size, bits, dtype)


def make_random_codes(rng, N, K, group_size=64, bits=4, dtype="bf16"):
    """Random packed codes + uniform scales/biases (bench/test_dispatch.py:34-42 style)."""
    w = rng.integers(0, 2**32, size=(N, K * bits // 32), dtype=np.uint64).astype(np.uint32)
    s = O.to_half(rng.uniform(0, 0.02, size=(N, K // group_size)), dtype)
    b = O.to_half(rng.uniform(-0.005, 0.005, size=(N, K // group_size)), dtype)
    return w, s, b


def make_x(rng, M, K, dtype="bf16", scale=1.0):
    return O.to_half(rng.normal(0, 1, size=(M, K)) * scale, dtype)


def check_close(got_half: np.ndarray, ref_f32: np.ndarray, dtype: str, what: str = ""):
    got = O.from_half(got_half, dtype).astype(np.float64)
    ref = ref_f32.astype(np.float64)
    nmax = O.normalized_max_error(got, ref)
    mae = O.mean_abs_error(got, ref)
    floor = O.mean_abs_error(O.from_half(O.to_half(ref_f32, dtype), dtype), ref)
    scale = max(1.0, float(np.abs(ref).mean())) if ref.size else 1.0
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert nmax <= 1e-2, f"{what}: normalised max error {nmax:.3e} > 1e-2"
    assert mae <= floor + 1e-3 * scale, f"{what}: MAE {mae:.3e} > {floor:.3e} + 1e-3*{scale:.2f}"
    return nmax, mae
