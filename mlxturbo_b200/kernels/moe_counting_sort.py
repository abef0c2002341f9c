"""Deterministic counting sort of MoE rows by expert
(mlxturbo/kernels/moe_counting_sort.py: hist -> exclusive scan -> in-order
scatter, no atomics in the output order).

``sort_rows(ids, n_experts, top_k)`` returns ``(order, idx_s, row_src, inv,
tables)`` like the reference: order = stable argsort(ids), idx_s = ids[order],
row_src = order // top_k, inv = argsort(order), and tables =
``segment_tables(counts, bm, mix_threshold)``.  Unlike the reference's
argsort chain the sort is stable, so the same input gives the same arrays on
every run.
"""

from __future__ import annotations

import torch

from .. import _lib
from ..ops import _contig, _stream, workspace
from . import _fire
from . import moe_grouped_gemm as mgg

MAX_EXPERTS = 16384


def eligible(ids: torch.Tensor, n_experts: int) -> bool:
    return ids.is_cuda and ids.dim() == 1 and 0 < n_experts <= MAX_EXPERTS


def sort_rows(ids: torch.Tensor, n_experts: int, top_k: int, bm: int = mgg.BM, mix_threshold: int | None = 48,
              with_tables: bool = True):
    if not eligible(ids, n_experts):
        raise ValueError("sort_rows: ids must be a 1-D CUDA tensor and 0 < n_experts <= 16384")
    _fire.bump("moe_counting_sort")
    ids = _contig(ids.to(torch.int32))
    M = ids.shape[0]
    dev = ids.device
    order, idx_s, row_src, inv = (torch.empty(M, dtype=torch.int32, device=dev) for _ in range(4))
    lib = _lib.load()
    ws_bytes = int(lib.qmm_sort_workspace_size(M, n_experts))
    ws = workspace(dev, ws_bytes)
    rc = lib.qmm_sort_rows(ids.data_ptr(), M, n_experts, top_k, order.data_ptr(), idx_s.data_ptr(), row_src.data_ptr(),
                           inv.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(rc, "sort_rows")
    if not with_tables:  # the caller builds its own tables (mgg.gather_tables)
        return order, idx_s, row_src, inv, None
    counts = mgg.counts_from_sorted_ids(idx_s, n_experts)
    tables = mgg.segment_tables(counts, bm=bm, mix_threshold=mix_threshold)
    return order, idx_s, row_src, inv, tables


__all__ = ["MAX_EXPERTS", "eligible", "sort_rows"]
