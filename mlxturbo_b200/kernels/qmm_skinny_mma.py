"""Skinny bf16 quantized matmul with explicit implementations
(mlxturbo/kernels/qmm_skinny_mma.py:1-249, _qmm_skinny_mma_source.py:9-40,
_qmm_e120_source.py:6-71).

``qmm_skinny_mma(x, w, scales, biases, group_size=64, bits=4, *,
implementation="v5", use_table=None)`` keeps the reference's signature, its
two implementation names and its ValueError checks:

- ``"v5"``: bf16, M = 6..16, N a multiple of 8, K a multiple of 64.
- ``"e120_v4"``: bf16, M = 2..9, N a multiple of 8, K a multiple of 512;
  ``use_table`` chose the Metal kernel's Sigma(x) table and is only valid here.

Both names run the B200 decode kernel (warp-level tensor-core MMA over the
whole M <= 16 window), so the implementation argument selects a contract,
not a different arithmetic.  Outside a contract the reference hands the call
to stock MLX (qmm_skinny_mma.py:151-152, 177-178); here that is
``ops.quantized_matmul``.
"""

from __future__ import annotations

import torch

from .. import ops
from . import _fire

GROUP_SIZE = 64
BITS = 4
M_MIN = 6
M_MAX = 16
MMA_TILE = 8
SPLIT_K = 8
THREADGROUP = (32, SPLIT_K, 1)

E120_M_MIN = 2
E120_M_MAX = 9
E120_BLOCK_SIZE = 512
E120_MINIMUM_TABLE_WIDTH = 4

V5_IMPLEMENTATION = "v5"
E120_V4_IMPLEMENTATION = "e120_v4"
_IMPLEMENTATIONS = frozenset((V5_IMPLEMENTATION, E120_V4_IMPLEMENTATION))


def eligible_layout(m: int, k: int, n: int, w_shape, scales_shape, biases_shape, group_size: int, bits: int) -> bool:
    """The v5 layout contract (_qmm_skinny_mma_source.py:18-39)."""
    if group_size != GROUP_SIZE or bits != BITS:
        return False
    if not (M_MIN <= m <= M_MAX) or k <= 0 or n <= 0:
        return False
    if k % GROUP_SIZE or n % MMA_TILE:
        return False
    if tuple(w_shape) != (n, k * bits // 32):
        return False
    groups = k // group_size
    return tuple(scales_shape) == (n, groups) and tuple(biases_shape) == (n, groups)


def e120_eligible_layout(m: int, k: int, n: int, w_shape, scales_shape, biases_shape, group_size: int,
                         bits: int) -> bool:
    """The E120 layout contract (_qmm_e120_source.py:50-71)."""
    if group_size != GROUP_SIZE or bits != BITS:
        return False
    if not (E120_M_MIN <= m <= E120_M_MAX) or k <= 0 or n <= 0:
        return False
    if k % E120_BLOCK_SIZE or n % 8:
        return False
    if tuple(w_shape) != (n, k * bits // 32):
        return False
    groups = k // group_size
    return tuple(scales_shape) == (n, groups) and tuple(biases_shape) == (n, groups)


def _common_eligible(x, w, scales, biases) -> bool:
    if not (isinstance(x, torch.Tensor) and x.is_cuda) or x.dtype != torch.bfloat16:
        return False
    if w.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
        return False
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        return False
    return x.dim() == w.dim() == scales.dim() == biases.dim() == 2


def _eligible(layout, x, w, scales, biases, group_size: int, bits: int) -> bool:
    if not _common_eligible(x, w, scales, biases):
        return False
    m, k = x.shape
    return layout(m, k, w.shape[0], tuple(w.shape), tuple(scales.shape), tuple(biases.shape), group_size, bits)


def qmm_skinny_mma(x, w, scales, biases, group_size: int = GROUP_SIZE, bits: int = BITS, *,
                   implementation: str = V5_IMPLEMENTATION, use_table: bool | None = None) -> torch.Tensor:
    """x [M, K] @ dequant(w [N, K]).T -> [M, N] bf16."""
    if implementation not in _IMPLEMENTATIONS:
        choices = ", ".join(sorted(_IMPLEMENTATIONS))
        raise ValueError(f"implementation must be one of {choices}, got {implementation!r}")
    if implementation == V5_IMPLEMENTATION and use_table is not None:
        raise ValueError("use_table is only valid with implementation='e120_v4'")
    layout = eligible_layout if implementation == V5_IMPLEMENTATION else e120_eligible_layout
    if _eligible(layout, x, w, scales, biases, group_size, bits):
        _fire.bump(f"qmm_skinny_mma_{implementation}")
    return ops.quantized_matmul(x, w, scales, biases, transpose=True, group_size=group_size, bits=bits)


__all__ = ["E120_V4_IMPLEMENTATION", "M_MAX", "M_MIN", "V5_IMPLEMENTATION", "qmm_skinny_mma"]
