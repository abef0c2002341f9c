"""Multi-row decode qmv with per-row single-call bits
(mlxturbo/kernels/qmv_small_m.py:61-335).

``qmv_small_m(x, w, scales, biases, group_size, bits, nsg, rps)`` is a drop-in
for ``mx.quantized_matmul(x, w, scales, biases, transpose=True)`` at M = 1..8
whose every output row has the bits of the M = 1 call on that row alone (the
reference's guarantee, bench/test_qmm_smallm.py:68-84).

On B200 that guarantee comes from the decode kernel itself: for M <= 8 its
schedule (row tiles, K segments, reduction order) is a function of (N, K)
only, and the activation rows are independent columns of one MMA n-tile.  So
this module only keeps the reference's eligibility contract and names; the
work is ``ops.quantized_matmul``.  ``nsg``/``rps`` (simdgroups per
threadgroup, rows per simdgroup of the Metal kernel) are accepted for call
compatibility and change nothing here.
"""

from __future__ import annotations

import torch

from .. import ops
from . import _fire

GROUP_SIZE = 64
BITS = 4
PACK_FACTOR = 8  # 32 / bits
PACKS_PER_THREAD = 2
VALUES_PER_THREAD = PACK_FACTOR * PACKS_PER_THREAD  # 16
SIMD_SIZE = 32
BLOCK_SIZE = VALUES_PER_THREAD * SIMD_SIZE  # 512
M_MIN = 1
M_MAX = 8
NUM_SIMDGROUPS = 2
RESULTS_PER_SIMDGROUP = 4

_HALF = (torch.bfloat16, torch.float16)
_U32 = (torch.int32, getattr(torch, "uint32", torch.int32))


def eligible(x, w, scales, biases, group_size: int, bits: int, m_min: int = M_MIN, m_max: int = M_MAX) -> bool:
    """The reference's shape/dtype contract (qmv_small_m.py:237-286): 4-bit g64,
    bf16/fp16 with matching scales/biases, 2-D operands, K a multiple of the
    512-value block, N a multiple of 8, m_min <= M <= m_max."""
    if not (isinstance(x, torch.Tensor) and x.is_cuda):
        return False
    if bits != BITS or group_size != GROUP_SIZE:
        return False
    if x.dtype not in _HALF or scales.dtype != x.dtype or biases.dtype != x.dtype:
        return False
    if w.dtype not in _U32:
        return False
    if x.dim() != 2 or w.dim() != 2 or scales.dim() != 2 or biases.dim() != 2:
        return False
    M, K = x.shape
    N = w.shape[0]
    if not (m_min <= M <= m_max):
        return False
    if group_size % VALUES_PER_THREAD or K % BLOCK_SIZE:
        return False
    if N % (NUM_SIMDGROUPS * RESULTS_PER_SIMDGROUP):
        return False
    if w.shape[1] != K * BITS // 32:
        return False
    n_groups = K // group_size
    return tuple(scales.shape) == (N, n_groups) and tuple(biases.shape) == (N, n_groups)


def qmv_small_m(x, w, scales, biases, group_size: int = GROUP_SIZE, bits: int = BITS, nsg: int = NUM_SIMDGROUPS,
                rps: int = RESULTS_PER_SIMDGROUP) -> torch.Tensor:
    """x [M, K] (M <= 8) -> [M, N] in x's dtype; each row equals its M = 1 call.

    Outside the contract the reference hands the call to stock MLX
    (qmv_small_m.py:308-322); here the same call goes to ``ops.quantized_matmul``,
    which raises on operands no kernel supports.
    """
    del nsg, rps
    if eligible(x, w, scales, biases, group_size, bits):
        _fire.bump("qmv_small_m")
    return ops.quantized_matmul(x, w, scales, biases, transpose=True, group_size=group_size, bits=bits)


__all__ = ["BLOCK_SIZE", "M_MAX", "M_MIN", "eligible", "qmv_small_m"]
