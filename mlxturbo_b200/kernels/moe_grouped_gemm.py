"""Expert-segmented grouped quantized matmul
(mlxturbo/kernels/moe_grouped_gemm.py: counts_from_sorted_ids :818-827,
segment_tables :829-855, n_tiles_max :858-867, segmented_eligible :870-910,
qmm_segmented :913-1065).

``qmm_segmented`` computes ``mx.gather_qmm(..., transpose=True,
sorted_indices=True)`` over rows sorted by expert, with the reference's
``row_src`` gather fold and ``row_dst``/``row_scale`` store epilogue.  The
tile arguments of the reference (bm, wm, bn, bk, frag_skip, mix_threshold)
are accepted for call compatibility; on B200 the kernel's tiling is its own
and none of them changes a result (each output row is a row-local dot
product).  Tables are built on the device; nothing syncs with the host.
"""

from __future__ import annotations

import torch

from .. import _lib
from ..ops import _contig, _dtype_code, _stream, workspace
from . import _fire

GROUP_SIZE = 64
BITS = 4
BM = 32
BM16 = 16
BN = 32
BK = 32
WM = 2
WM16 = 1
WN = 2


def counts_from_sorted_ids(ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    """(num_experts,) int32 row counts of expert ids (sorted or not)."""
    ids = _contig(ids.reshape(-1).to(torch.int32))
    counts = torch.empty(num_experts, dtype=torch.int32, device=ids.device)
    rc = _lib.load().qmm_segment_tables(ids.data_ptr(), ids.numel(), num_experts, BM, 0, counts.data_ptr(), None, None,
                                        _stream(ids.device))
    _lib.check(rc, "counts_from_sorted_ids")
    return counts


def segment_tables(counts: torch.Tensor, bm: int = BM, mix_threshold: int | None = None):
    """(row_start, tile_prefix), both (E+1,) int32, from per-expert counts."""
    counts = _contig(counts.to(torch.int32))
    E = counts.numel()
    row_start = torch.empty(E + 1, dtype=torch.int32, device=counts.device)
    tile_prefix = torch.empty(E + 1, dtype=torch.int32, device=counts.device)
    rc = _lib.load().qmm_segment_tables_from_counts(counts.data_ptr(), E, int(bm), int(mix_threshold or 0),
                                                    row_start.data_ptr(), tile_prefix.data_ptr(),
                                                    _stream(counts.device))
    _lib.check(rc, "segment_tables")
    return row_start, tile_prefix


def n_tiles_max(num_rows: int, num_experts: int, bm: int = BM) -> int:
    """Static bound on the tile count: floor(M/bm) + min(E, M)."""
    return num_rows // bm + min(num_experts, num_rows)


def segmented_eligible(x, w, scales, biases, group_size: int = GROUP_SIZE, bits: int = BITS) -> bool:
    """Whether qmm_segmented takes these operands (shape/dtype contract)."""
    if bits not in (4, 8) or group_size not in (32, 64, 128):
        return False
    if x.dim() != 2 or w.dim() != 3 or scales.dim() != 3 or biases.dim() != 3:
        return False
    if x.dtype not in (torch.bfloat16, torch.float16):
        return False
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        return False
    if w.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
        return False
    K = x.shape[1]
    E, N = w.shape[0], w.shape[1]
    if K % group_size or w.shape[2] * 32 != K * bits:
        return False
    return tuple(scales.shape) == (E, N, K // group_size) and tuple(biases.shape) == tuple(scales.shape)


def qmm_segmented(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                  segments: torch.Tensor | None, *, num_experts: int | None = None, segments_are: str = "auto",
                  tables=None, frag_skip: bool = False, bm: int = BM, wm: int | None = None,
                  mix_threshold: int | None = None, group_size: int = GROUP_SIZE, bits: int = BITS,
                  row_dst: torch.Tensor | None = None, row_scale: torch.Tensor | None = None,
                  row_src: torch.Tensor | None = None, bn: int = BN, bk: int = BK) -> torch.Tensor:
    """gather_qmm over expert-sorted rows -> (M, N), M = len(row_src) or x rows."""
    del frag_skip, wm, bn, bk  # tiling knobs of the Metal kernel; no effect on results here
    _fire.bump("moe_grouped_gemm_segmented")
    K = x.shape[1]
    M = x.shape[0] if row_src is None else row_src.shape[0]
    E, N = w.shape[0], w.shape[1]
    if num_experts is not None and num_experts != E:
        raise ValueError(f"num_experts={num_experts} does not match w's {E}")
    if not segmented_eligible(x, w, scales, biases, group_size, bits):
        raise NotImplementedError("qmm_segmented: operands outside the supported contract")
    if tables is None:
        kind = segments_are
        if kind == "auto":
            if segments.numel() == M:
                kind = "ids"
            elif segments.numel() == E:
                kind = "counts"
            else:
                raise ValueError(f"segments has {segments.numel()} elements, neither M={M} nor E={E}")
        if kind == "ids":
            counts = counts_from_sorted_ids(segments, E)
        elif kind == "counts":
            counts = segments
        else:
            raise ValueError(f"segments_are={segments_are!r}")
        tables = segment_tables(counts, bm=bm, mix_threshold=mix_threshold)
    row_start = _contig(tables[0].to(torch.int32))
    if (row_dst is None) != (row_scale is None):
        raise ValueError("row_dst and row_scale go together")
    if row_dst is not None and (row_dst.shape != (M,) or row_scale.shape != (M,)):
        raise ValueError("row_dst/row_scale must have shape (M,)")
    dev = x.device
    x, w, scales, biases = _contig(x), _contig(w), _contig(scales), _contig(biases)
    rs = None if row_src is None else _contig(row_src.to(torch.int32))
    rd = None if row_dst is None else _contig(row_dst.to(torch.int32))
    sc = None if row_scale is None else _contig(row_scale.to(torch.float32))
    out = torch.empty((M, N), dtype=x.dtype, device=dev)
    lib = _lib.load()
    ws = workspace(dev, int(lib.qmm_segmented_workspace_size(M, E)), zeroed=True)  # tile counters first
    rc = lib.qmm_segmented(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), row_start.data_ptr(),
                           None if rs is None else rs.data_ptr(), None if rd is None else rd.data_ptr(),
                           None if sc is None else sc.data_ptr(), out.data_ptr(), M, x.shape[0], E, N, K, group_size,
                           bits, _dtype_code(x), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(rc, "qmm_segmented")
    return out


class GatherTables:
    """Segment tables of expert-sorted rows, built once for several gather_run calls.

    They live in the device workspace they were built in and stay valid until
    the next gather on that workspace (an MoE block: tables, gate/up, down).
    """

    def __init__(self, ws: torch.Tensor, rows: int, num_experts: int):
        self.ws, self.rows, self.num_experts = ws, rows, num_experts


def gather_tables(idx_s: torch.Tensor, num_experts: int) -> GatherTables:
    """Tables for rows whose expert ids `idx_s` (int32/uint32 [rows]) are non-decreasing."""
    idx_s = _contig(idx_s.reshape(-1).to(torch.int32) if idx_s.dtype != torch.int32 else idx_s.reshape(-1))
    rows = idx_s.numel()
    lib = _lib.load()
    ws = workspace(idx_s.device, int(lib.qmm_segmented_workspace_size(rows, num_experts)), zeroed=True)
    rc = lib.qmm_gather_tables(idx_s.data_ptr(), rows, num_experts, ws.data_ptr(), ws.numel(), _stream(idx_s.device))
    _lib.check(rc, "gather_tables")
    return GatherTables(ws, rows, num_experts)


ROUTE_MAX_ROWS, ROUTE_MAX_EXPERTS = 16384, 1024


def moe_route(ids: torch.Tensor, num_experts: int, top_k: int):
    """The counting sort and the gather tables in one launch (decode / verify batches).

    ``ids`` int32 [rows] expert ids in token-major order.  Returns ``(order,
    idx_s, row_src, inv, tables)`` -- the arrays of
    ``moe_counting_sort.sort_rows`` bit for bit and the tables of
    ``gather_tables(idx_s)`` -- or None when the batch is outside the one-launch
    route (more than 16384 rows or 1024 experts).
    """
    ids = ids.reshape(-1)
    rows = ids.numel()
    if not ids.is_cuda or rows == 0 or rows > ROUTE_MAX_ROWS or not 0 < num_experts <= ROUTE_MAX_EXPERTS:
        return None
    ids = _contig(ids if ids.dtype == torch.int32 else ids.to(torch.int32))
    dev = ids.device
    out = torch.empty((4, rows), dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, int(lib.qmm_segmented_workspace_size(rows, num_experts)), zeroed=True)
    p = out.data_ptr()
    rc = lib.qmm_moe_route(ids.data_ptr(), rows, num_experts, top_k, p, p + 4 * rows, p + 8 * rows, p + 12 * rows,
                           ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(rc, "moe_route")
    _fire.bump("moe_route")
    return out[0], out[1], out[2], out[3], GatherTables(ws, rows, num_experts)


def gather_run(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, tables: GatherTables, *,
               row_src: torch.Tensor | None = None, row_dst: torch.Tensor | None = None,
               row_scale: torch.Tensor | None = None, glu: bool = False, group_size: int = GROUP_SIZE,
               bits: int = BITS) -> torch.Tensor:
    """The gathered matmul on prebuilt tables -> (rows, N) (or (rows, N/2) with glu).

    glu: w/scales/biases are a fused gate/up bank interleaved per 16-row block
    (``nn.SwitchGLU.fused_gate_up``) and the result is silu(gate) * up.
    Raises NotImplementedError when the problem exceeds the kernel's tile
    counters (use qmm_segmented then).
    """
    rows, E = tables.rows, tables.num_experts
    N, K = w.shape[1], x.shape[-1]
    dev = x.device
    # rows of a wider buffer (an expert-parallel receive buffer, ids after each
    # row) are read in place
    x_stride = 0
    if x.dim() == 2 and x.stride(1) == 1 and x.stride(0) != K and x.stride(0) >= K and x.stride(0) % 8 == 0 \
            and x.data_ptr() % 16 == 0:
        x_stride = x.stride(0)
    else:
        x = _contig(x)
    w, scales, biases = _contig(w), _contig(scales), _contig(biases)
    rs = None if row_src is None else _contig(row_src.to(torch.int32) if row_src.dtype != torch.int32 else row_src)
    rd = None if row_dst is None else _contig(row_dst.to(torch.int32) if row_dst.dtype != torch.int32 else row_dst)
    sc = None if row_scale is None else _contig(row_scale.to(torch.float32))
    out = torch.empty((rows, N // 2 if glu else N), dtype=x.dtype, device=dev)
    lib = _lib.load()
    x_rows = x.shape[0] if x.dim() == 2 else x.numel() // K
    rc = lib.qmm_gather_run(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                            None if rs is None else rs.data_ptr(), None if rd is None else rd.data_ptr(),
                            None if sc is None else sc.data_ptr(), out.data_ptr(), rows, x_rows, x_stride, E, N, K,
                            group_size,
                            bits, _dtype_code(x), int(glu), tables.ws.data_ptr(), tables.ws.numel(), _stream(dev))
    _lib.check(rc, "gather_run")
    return out


def enabled() -> bool:
    return True


__all__ = [
    "BM", "BM16", "BN", "BK", "GatherTables", "counts_from_sorted_ids", "enabled", "gather_run", "gather_tables",
    "moe_route",
    "n_tiles_max", "qmm_segmented", "segment_tables", "segmented_eligible",
]
