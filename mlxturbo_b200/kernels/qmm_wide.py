"""Prefill quantized matmul with a wide token tile (mlxturbo/kernels/qmm_wide.py:93-502).

``qmm_wide(x, w, scales, biases, *, tile=Tile(64, 32, 32, 2, 2), group_size=64,
bits=4)`` computes ``mx.quantized_matmul(x, w, scales, biases,
transpose=True)`` for prefill widths by dequantising weight tiles once and
reusing them across many activation rows.

The reference sweeps Metal threadgroup tiles (``Tile``: bm activation rows x
bn weight rows x bk K values, wm x wn simdgroups).  On B200 the kernel is the
tcgen05 prefill kernel (csrc/prefill.cu): 128 weight rows x 128 or 256
tokens per CTA, fixed by the tensor-core instruction shape and TMEM, chosen
by M.  The reference's tile type, its candidate list and its validity rules
(``tile_ok``) are kept so callers and tests written against them behave the
same: an invalid tile still raises ``ValueError``.  A valid tile does not
change the B200 kernel, so every valid tile gives the same bits, which is the
reference's own all-tiles gate (bench/test_qmm_wide_shapes.py:82-100).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from . import _fire

GROUP_SIZE = 64
BITS = 4
SIMD_SIZE = 32
FRAG = 8


@dataclass(frozen=True)
class Tile:
    """A reference threadgroup tile: bm x bn outputs, bk K step, wm x wn simdgroups."""

    bm: int
    bn: int
    bk: int
    wm: int
    wn: int
    xreads: int = 0

    @property
    def threads(self) -> int:
        return self.wm * self.wn * SIMD_SIZE

    @property
    def x_reads(self) -> int:
        return self.xreads or ((self.bk * self.bm) // self.threads)

    @property
    def name(self) -> str:
        base = f"m{self.bm}n{self.bn}k{self.bk}w{self.wm}x{self.wn}"
        return base if not self.xreads else f"{base}r{self.xreads}"

    @property
    def tgp_bytes(self) -> int:
        """bf16 threadgroup bytes of the Metal kernel (Xs + Ws, padded K)."""
        return (self.bm + self.bn) * (self.bk + 8) * 2

    @property
    def accum_regs(self) -> int:
        tm = self.bm // (FRAG * self.wm)
        tn = self.bn // (FRAG * self.wn)
        return tm * tn * 2


STOCK = Tile(32, 32, 32, 2, 2)

TILES: dict[str, Tile] = {t.name: t for t in [
    STOCK,
    Tile(64, 32, 32, 2, 2),
    Tile(64, 32, 32, 2, 2, xreads=8),
    Tile(64, 32, 32, 4, 2),
    Tile(64, 64, 32, 2, 2),
    Tile(64, 64, 32, 2, 4),
    Tile(64, 64, 32, 4, 2),
    Tile(128, 32, 32, 4, 2),
    Tile(128, 64, 32, 4, 2),
    Tile(64, 32, 64, 2, 2, xreads=8),
    Tile(64, 64, 64, 2, 4, xreads=8),
]}


def tile_ok(tile: Tile, K: int, N: int, group_size: int = GROUP_SIZE, bits: int = BITS) -> str | None:
    """Why `tile` is not a valid reference tile for (K, N), or None (qmm_wide.py:345-372)."""
    if tile.bm % (FRAG * tile.wm) or tile.bn % (FRAG * tile.wn):
        return "BM/BN not divisible by the 8-wide fragment x WM/WN"
    if tile.bk < SIMD_SIZE or tile.bk % SIMD_SIZE:
        return "BK is not a multiple of the SIMD width"
    if tile.bk > group_size or group_size % tile.bk:
        return "BK exceeds or does not divide group_size"
    if K % tile.bk:
        return f"K={K} is not a multiple of BK={tile.bk}"
    pack_factor = 8 // bits
    bcols_packed = tile.bk // pack_factor
    if (bcols_packed * tile.bn) % tile.threads:
        return "the W loader's BCOLS_PACKED * BN is not a multiple of the thread count"
    if bcols_packed * tile.bn < tile.threads:
        return "the W tile is smaller than the thread count"
    if (tile.bk * tile.bm) % tile.threads:
        return "the X tile is not a multiple of the thread count"
    if tile.bk % tile.x_reads or (tile.threads * tile.x_reads) % tile.bk:
        return "XREADS does not divide BK"
    if tile.tgp_bytes > 32 * 1024:
        return f"threadgroup memory {tile.tgp_bytes} B exceeds 32 KB"
    if tile.threads > 1024:
        return "more than 1024 threads"
    return None


_STOCK_QMV_MAX_ROWS = 13
_STOCK_SPLITK_TILES = 256
_STOCK_SPLITK_MIN_K = 128


def stock_bit_matches(M: int, K: int, N: int) -> bool:
    """Whether stock MLX picks ``qmm_t`` for this shape (qmm_wide.py:380-397):
    M >= 13 and either K < 128 or at least 256 32x32 output tiles."""
    if M < _STOCK_QMV_MAX_ROWS:
        return False
    if K < _STOCK_SPLITK_MIN_K:
        return True
    tiles = ((M + 31) // 32) * ((N + 31) // 32)
    return tiles >= _STOCK_SPLITK_TILES


def eligible(x, w, scales, biases, tile: Tile, group_size: int = GROUP_SIZE, bits: int = BITS) -> bool:
    """Shape/dtype contract of qmm_wide (qmm_wide.py:423-453)."""
    if bits != BITS:
        return False
    if x.dim() != 2 or w.dim() != 2 or scales.dim() != 2 or biases.dim() != 2:
        return False
    if x.dtype not in (torch.bfloat16, torch.float16):
        return False
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        return False
    if w.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
        return False
    K = x.shape[1]
    N = w.shape[0]
    if K % group_size or w.shape[1] != K * bits // 32:
        return False
    groups = K // group_size
    if tuple(scales.shape) != (N, groups) or tuple(biases.shape) != (N, groups):
        return False
    return tile_ok(tile, K, N, group_size, bits) is None


def qmm_wide(x, w, scales, biases, *, tile: Tile = Tile(64, 32, 32, 2, 2), group_size: int = GROUP_SIZE,
             bits: int = BITS) -> torch.Tensor:
    """x (M, K), w (N, K*bits/32) packed, scales/biases (N, K/group_size) -> (M, N).

    Runs the tcgen05 prefill kernel at any M (it is the wide-tile path even
    for a handful of rows, as the reference's is).
    """
    why = tile_ok(tile, x.shape[1], w.shape[0], group_size, bits)
    if why is not None:
        raise ValueError(f"tile {tile.name} is not valid: {why}")
    _fire.bump(f"qmm_wide_{tile.name}")
    tokens = 128 if x.shape[0] <= 128 else 256
    return ops.prefill_explicit(x, w, scales, biases, group_size=group_size, bits=bits, tokens_per_cta=tokens)


__all__ = ["STOCK", "TILES", "Tile", "eligible", "qmm_wide", "stock_bit_matches", "tile_ok"]
