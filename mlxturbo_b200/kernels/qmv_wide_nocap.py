"""Single-tile wide qmv for verify widths (mlxturbo/kernels/qmv_wide_nocap.py:58-288).

``qmv_wide_nocap(x, w, scales, biases, group_size=64, bits=4, m_min=6)`` is a
drop-in for ``mx.quantized_matmul(..., transpose=True)`` at M = m_min..12 that
reads the quantized weights once per call instead of ceil(M/5) times (stock
MLX's ``qmv_wide`` tiling).

On B200 the decode kernel already reads each weight tile once for any
M <= 16 (all activation rows ride in one or two MMA n-tiles), so this module
keeps the reference's eligibility contract and names and runs
``ops.quantized_matmul``.
"""

from __future__ import annotations

import torch

from .. import ops
from . import _fire

GROUP_SIZE = 64
BITS = 4
M_MIN = 6
M_MAX = 12
K_LANES = 8
NUM_SIMDGROUPS = 2
RESULTS_PER_SIMDGROUP = 32 // K_LANES
ROWS_PER_TG = RESULTS_PER_SIMDGROUP * NUM_SIMDGROUPS
SUB = 8

_HALF = (torch.bfloat16, torch.float16)
_U32 = (torch.int32, getattr(torch, "uint32", torch.int32))


def _eligible(x, w, scales, biases, group_size: int, bits: int, m_min: int = M_MIN) -> bool:
    """The reference's contract (qmv_wide_nocap.py:204-237): 4-bit g64,
    bf16/fp16 with matching scales/biases, 2-D operands, m_min <= M <= 12,
    K a multiple of 64."""
    if not (isinstance(x, torch.Tensor) and x.is_cuda):
        return False
    if group_size != GROUP_SIZE or bits != BITS:
        return False
    if x.dtype not in _HALF or scales.dtype != x.dtype or biases.dtype != x.dtype:
        return False
    if w.dtype not in _U32:
        return False
    if x.dim() != 2 or w.dim() != 2 or scales.dim() != 2 or biases.dim() != 2:
        return False
    M, K = x.shape
    N = w.shape[0]
    if not (m_min <= M <= M_MAX) or K % GROUP_SIZE:
        return False
    if w.shape[1] != K * BITS // 32:
        return False
    n_groups = K // GROUP_SIZE
    return tuple(scales.shape) == (N, n_groups) and tuple(biases.shape) == (N, n_groups)


def qmv_wide_nocap(x, w, scales, biases, group_size: int = 64, bits: int = 4, m_min: int = M_MIN) -> torch.Tensor:
    """x [M, K] -> [M, N] in x's dtype; weights read once per call.

    Outside the contract the reference delegates to stock MLX
    (qmv_wide_nocap.py:272-275); here that is ``ops.quantized_matmul`` too.
    """
    if _eligible(x, w, scales, biases, group_size, bits, m_min):
        _fire.bump("qmv_wide_nocap")
    return ops.quantized_matmul(x, w, scales, biases, transpose=True, group_size=group_size, bits=bits)


__all__ = ["M_MAX", "M_MIN", "qmv_wide_nocap"]
