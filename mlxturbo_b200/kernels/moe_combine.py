"""MoE combine: unsort + router weight + top_k sum in one pass
(mlxturbo/kernels/moe_combine.py:1-60, 67-189).

    y[t, n] = sum_k w[t*top_k + k] * out_sorted[inv[t*top_k + k], n]

fp32 accumulation in k order, one rounding at the store.
"""

from __future__ import annotations

import torch

from .. import _lib
from ..ops import _contig, _dtype_code, _stream
from . import _fire

VEC = 8  # columns per thread (16-byte loads/stores)


def eligible(out_sorted: torch.Tensor, rows: int, top_k: int) -> bool:
    """A CUDA (R, N) bf16/fp16 source; R is rows*top_k, or more when the results
    sit in a larger buffer (inv entries past R are skipped)."""
    return (out_sorted.is_cuda and out_sorted.dim() == 2 and out_sorted.dtype in (torch.bfloat16, torch.float16)
            and out_sorted.shape[0] >= rows * top_k)


def combine(out_sorted: torch.Tensor, inv: torch.Tensor, w: torch.Tensor, rows: int, top_k: int,
            chained: bool = False) -> torch.Tensor:
    """(rows*top_k, N) sorted expert outputs -> (rows, N) token outputs.

    ``chained``: the previous operation on the stream is this package's own
    gathered matmul (qmm_moe_combine_chained: programmatic dependent launch).
    """
    if not eligible(out_sorted, rows, top_k):
        raise ValueError("combine: out_sorted must be a CUDA (>= rows*top_k, N) bf16/fp16 tensor")
    _fire.bump("moe_combine")
    N = out_sorted.shape[1]
    out_sorted = _contig(out_sorted)
    inv = _contig(inv.to(torch.int32) if inv.dtype not in (torch.int32, torch.uint32) else inv)
    w = _contig(w.to(torch.float32))
    y = torch.empty((rows, N), dtype=out_sorted.dtype, device=out_sorted.device)
    lib = _lib.load()
    entry = lib.qmm_moe_combine_chained if chained else lib.qmm_moe_combine_rows
    rc = entry(out_sorted.data_ptr(), out_sorted.shape[0], inv.data_ptr(), w.data_ptr(), y.data_ptr(), rows, top_k, N,
               _dtype_code(out_sorted), _stream(out_sorted.device))
    _lib.check(rc, "moe_combine")
    return y


__all__ = ["VEC", "combine", "eligible"]
