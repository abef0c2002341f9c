"""numpy/ctypes front end of the CPU oracle (qmm_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker, and by bench.py's CPU legs.  The product package never imports it.

16-bit floats travel as numpy ``uint16`` bit patterns; ``dtype`` is "bf16" or
"f16".  Every function states the reference code it restates (see the C file).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_DT = {"bf16": 0, "f16": 1}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int

_SIGS = {
    "oracle_unpack_codes": [_p, _i64, _i64, _i, _p],
    "oracle_pack_codes": [_p, _i64, _i64, _i, _p],
    "oracle_dequantize": [_p, _p, _p, _i, _i64, _i64, _i, _i, _p],
    "oracle_quantize": [_p, _i64, _i64, _i, _i, _i, _p, _p, _p],
    "oracle_qmm_f32": [_p, _i, _i64, _i64, _p, _p, _p, _i64, _i, _i, _p, _i],
    "oracle_qmv_mlx_order": [_p, _i, _i64, _i64, _p, _p, _p, _i64, _p],
    "oracle_gather_qmm_f32": [_p, _i, _i64, _i64, _p, _p, _p, _i64, _i64, _i, _i, _p, _p, _i64, _p, _i],
    "oracle_sort_rows": [_p, _i64, _i64, _i, _p, _p, _p, _p],
    "oracle_segment_tables": [_p, _i64, _i, _i, _p, _p],
    "oracle_moe_combine": [_p, _i, _p, _p, _i64, _i, _i64, _p, _p],
    "oracle_f32_to_half_array": [_p, _i64, _i, _p],
    "oracle_half_to_f32_array": [_p, _i64, _i, _p],
    "oracle_num_threads": [],
}


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = _i if name == "oracle_num_threads" else None
    return _lib


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def num_threads() -> int:
    return lib().oracle_num_threads()


# --------------------------------------------------------------------------
# 16-bit float helpers
# --------------------------------------------------------------------------

def to_half(a: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    """fp32 -> bf16/f16 bit patterns (round to nearest even)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_f32_to_half_array(_ptr(a), a.size, _DT[dtype], _ptr(out))
    return out


def from_half(h: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().oracle_half_to_f32_array(_ptr(h), h.size, _DT[dtype], _ptr(out))
    return out


# --------------------------------------------------------------------------
# Layout and quantisation
# --------------------------------------------------------------------------

def unpack_codes(w: np.ndarray, K: int, bits: int) -> np.ndarray:
    """uint32 [N, K*bits/32] -> uint8 codes [N, K] (value k at bit k*bits)."""
    w = np.ascontiguousarray(w, dtype=np.uint32)
    N = w.shape[0]
    codes = np.empty((N, K), dtype=np.uint8)
    lib().oracle_unpack_codes(_ptr(w), N, K, bits, _ptr(codes))
    return codes


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    N, K = codes.shape
    w = np.empty((N, K * bits // 32), dtype=np.uint32)
    lib().oracle_pack_codes(_ptr(codes), N, K, bits, _ptr(w))
    return w


def dequantize(w, scales, biases, K: int, group_size: int, bits: int, dtype: str = "bf16") -> np.ndarray:
    """fp32 s*q + b, [N, K]."""
    w = np.ascontiguousarray(w, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    N = w.shape[0]
    out = np.empty((N, K), dtype=np.float32)
    lib().oracle_dequantize(_ptr(w), _ptr(scales), _ptr(biases), _DT[dtype], N, K, group_size, bits, _ptr(out))
    return out


def quantize(wf: np.ndarray, group_size: int = 64, bits: int = 4, dtype: str = "bf16"):
    """MLX affine quantisation of fp32 weights [N, K] -> (w, scales, biases)."""
    wf = np.ascontiguousarray(wf, dtype=np.float32)
    N, K = wf.shape
    assert K % group_size == 0 and (K * bits) % 32 == 0
    wq = np.empty((N, K * bits // 32), dtype=np.uint32)
    s = np.empty((N, K // group_size), dtype=np.uint16)
    b = np.empty((N, K // group_size), dtype=np.uint16)
    lib().oracle_quantize(_ptr(wf), N, K, group_size, bits, _DT[dtype], _ptr(wq), _ptr(s), _ptr(b))
    return wq, s, b


# --------------------------------------------------------------------------
# Matmuls
# --------------------------------------------------------------------------

def qmm(x, w, scales, biases, group_size: int = 64, bits: int = 4, dtype: str = "bf16",
        nthreads: int = 0) -> np.ndarray:
    """fp32 dequantise-then-matmul, y[M, N] fp32 (transpose=True)."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    lib().oracle_qmm_f32(_ptr(x), _DT[dtype], M, K, _ptr(w), _ptr(scales), _ptr(biases), N, group_size, bits,
                         _ptr(y), nthreads)
    return y


def qmv_mlx_order(x, w, scales, biases, dtype: str = "bf16") -> np.ndarray:
    """MLX qmv_fast lane order (4-bit, group 64, K % 512 == 0) -> T bits [M, N]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    assert K % 512 == 0
    y = np.empty((M, N), dtype=np.uint16)
    lib().oracle_qmv_mlx_order(_ptr(x), _DT[dtype], M, K, _ptr(np.ascontiguousarray(w, np.uint32)),
                               _ptr(np.ascontiguousarray(scales, np.uint16)),
                               _ptr(np.ascontiguousarray(biases, np.uint16)), N, _ptr(y))
    return y


def gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices, group_size: int = 64, bits: int = 4,
               dtype: str = "bf16", nthreads: int = 0) -> np.ndarray:
    """y[r] = x[lhs[r]] @ dequant(w[rhs[r]])^T, fp32 [rows, N]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint32)
    E, N = w.shape[0], w.shape[1]
    x_rows, K = x.shape
    rhs = np.ascontiguousarray(rhs_indices, dtype=np.int32)
    lhs = None if lhs_indices is None else np.ascontiguousarray(lhs_indices, dtype=np.int32)
    rows = rhs.shape[0]
    y = np.empty((rows, N), dtype=np.float32)
    lib().oracle_gather_qmm_f32(_ptr(x), _DT[dtype], x_rows, K, _ptr(w),
                                _ptr(np.ascontiguousarray(scales, np.uint16)),
                                _ptr(np.ascontiguousarray(biases, np.uint16)), E, N, group_size, bits,
                                _ptr(lhs), _ptr(rhs), rows, _ptr(y), nthreads)
    return y


# --------------------------------------------------------------------------
# MoE glue
# --------------------------------------------------------------------------

def sort_rows(ids, n_experts: int, top_k: int):
    """Stable counting sort -> (order, idx_s, row_src, inv), all uint32."""
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    M = ids.shape[0]
    outs = [np.empty((M,), dtype=np.uint32) for _ in range(4)]
    lib().oracle_sort_rows(_ptr(ids), M, n_experts, top_k, *[_ptr(o) for o in outs])
    return tuple(outs)


def segment_tables(counts, bm: int = 32, mix_threshold: int | None = None):
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    E = counts.shape[0]
    rs = np.empty((E + 1,), dtype=np.int32)
    tp = np.empty((E + 1,), dtype=np.int32)
    lib().oracle_segment_tables(_ptr(counts), E, bm, int(mix_threshold or 0), _ptr(rs), _ptr(tp))
    return rs, tp


def moe_combine(out_sorted, inv, wts, rows: int, top_k: int, dtype: str = "bf16"):
    """-> (y T bits [rows, N], y fp32 [rows, N])."""
    out_sorted = np.ascontiguousarray(out_sorted, dtype=np.uint16)
    N = out_sorted.shape[1]
    y = np.empty((rows, N), dtype=np.uint16)
    yf = np.empty((rows, N), dtype=np.float32)
    lib().oracle_moe_combine(_ptr(out_sorted), _DT[dtype], _ptr(np.ascontiguousarray(inv, np.uint32)),
                             _ptr(np.ascontiguousarray(wts, np.float32)), rows, top_k, N, _ptr(y), _ptr(yf))
    return y, yf


# --------------------------------------------------------------------------
# Error metrics used by every parity test (the reference's normalised form,
# bench/test_dispatch.py:66-73, and mean absolute error).
# --------------------------------------------------------------------------

def normalized_max_error(actual: np.ndarray, expected: np.ndarray) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    if e.size == 0:
        return 0.0
    return float(np.abs(a - e).max() / max(np.abs(e).max(), 1.0))


def mean_abs_error(actual: np.ndarray, expected: np.ndarray) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    if e.size == 0:
        return 0.0
    return float(np.abs(a - e).mean())
