"""MoE block folds around the expert-segmented quantized matmul.

Mirrors of the reference's MoE glue on the quantized-matmul path:

- ``moe_combine_fold(switch_mlp, x, idx, w)``, the SparseMoeBlock combine
  (mlxturbo/_vendor/qwen4_exp.py:1763-1806).  The router weight multiplies
  the SwiGLU output before ``down_proj``, and the top_k sum is taken on
  ``down_proj``'s output.  With ``idx.numel() >= MOE_COMBINE_SORT_MIN`` the
  (token, k) rows are sorted by expert first so every expert's rows are
  contiguous (``sorted_indices=True``).
- ``moe_fold_block(switch_mlp, x_rows, row_src, idx_s, order, w_flat)``, the
  down-epilogue hook (mlxturbo/fused.py:3220-3326).  gate/up run as one
  segmented GEMM each, with the x gather folded into the load (``row_src``).
  Then ``down_proj`` runs, followed by either the one-pass combine kernel
  (mode ``"combine"``: unsort, router weight, top_k sum) or a scattered
  store (mode ``"epi"``: ``row_dst``/``row_scale``, then the top_k sum).
- ``inv_perm(order)``, the inverse permutation by one scatter
  (mlxturbo/fused.py:3329-3336).
- ``fused_glu_block``: the same block for decode / verify batches.  Up to
  ``kernels.moe_decode_fused.MAX_PAIRS`` (token, expert) pairs it is one
  launch (``qmm_moe_glu_decode``: per-pair gate/up with the SwiGLU epilogue,
  a grid barrier, down with the weighted top_k sum); above that four launches
  (the counting sort and the segment tables in one route launch, one gathered
  matmul over the fused gate/up bank with the SwiGLU epilogue, down,
  combine); larger batches sort and build the tables in separate launches.  ``moe_combine_fold`` takes it whenever the down-epilogue hook does
  not take the call (``MLXTURBO_FUSED_GLU=0`` restores the
  projection-by-projection path).

The sort is the device counting sort (kernels/moe_counting_sort.py), which
is stable.  Expert tables are built on the device, and nothing here
synchronises with the host.
"""

from __future__ import annotations

import os

import torch

from .kernels import _fire
from .kernels import moe_combine as mc
from .kernels import moe_counting_sort as mcs
from .kernels import moe_decode_fused as mdf
from .kernels import moe_grouped_gemm as mgg

MOE_COMBINE_SORT_MIN = int(os.environ.get("MLXTURBO_SORT_MIN", "0") or 0) or 64
MOE_GEMM_MIN_ROWS = int(os.environ.get("MLXTURBO_MOE_GEMM_MIN_ROWS", "1024"))
MOE_GEMM_BM = 32
MOE_GEMM_MIX: int | None = None

_DOWN_EPI_ON = False
_FOLD_MODE = "combine"
_GATHER_FOLD_ON = True
# gate and up in one gathered launch with the SwiGLU epilogue (MLXTURBO_FUSED_GLU=0 restores
# the projection-by-projection path of the reference's block)
FUSED_GLU = os.environ.get("MLXTURBO_FUSED_GLU", "1") != "0"


def enable_moe_down_epilogue(mode: str | None = None, gather_fold: bool | None = None) -> None:
    """Route the sorted MoE path through ``moe_fold_block``.

    This is the switch of fused.py:3360-3396.  ``mode`` is ``"combine"``
    (default, env MLXTURBO_MOE_DOWN_EPI) or ``"epi"``; ``"off"`` disables.
    ``gather_fold`` (env MLXTURBO_MOE_GATHER_FOLD, default on) reads x rows
    through ``row_src`` inside the GEMM instead of gathering them first.
    """
    global _DOWN_EPI_ON, _FOLD_MODE, _GATHER_FOLD_ON
    if mode is None:
        mode = os.environ.get("MLXTURBO_MOE_DOWN_EPI", "combine").strip().lower() or "combine"
    if mode in ("off", "0", "none", "false", "no"):
        disable_moe_down_epilogue()
        return
    if mode not in ("combine", "epi"):
        raise ValueError(f"mode={mode!r} must be combine, epi or off")
    if gather_fold is None:
        gather_fold = os.environ.get("MLXTURBO_MOE_GATHER_FOLD", "1") not in ("0", "")
    _FOLD_MODE = mode
    _GATHER_FOLD_ON = bool(gather_fold)
    _DOWN_EPI_ON = True


def disable_moe_down_epilogue() -> None:
    global _DOWN_EPI_ON
    _DOWN_EPI_ON = False


def inv_perm(order: torch.Tensor) -> torch.Tensor:
    """The inverse of permutation ``order`` (== argsort(order)) by one scatter."""
    n = order.shape[0]
    idx = torch.arange(n, dtype=torch.int32, device=order.device)
    return torch.empty(n, dtype=torch.int32, device=order.device).scatter_(0, order.long(), idx)


def _proj_parts(proj):
    if proj.bias is not None or getattr(proj, "mode", "affine") != "affine":
        return None
    return proj.weight, proj.scales, proj.biases


def moe_fold_block(switch_mlp, x_rows: torch.Tensor, row_src: torch.Tensor, idx_s: torch.Tensor,
                   order: torch.Tensor, w_flat: torch.Tensor, *, tables=None, inv: torch.Tensor | None = None):
    """gate/up -> SwiGLU -> down over expert-sorted rows; (rows, hidden) or None.

    ``x_rows`` (rows, 1, K) is x before the gather; ``row_src`` (M,) the x row
    of sorted row s (order // top_k); ``idx_s`` (M,) sorted expert ids;
    ``order`` (M,) the stable argsort of the flat ids; ``w_flat`` (M,) fp32
    router weights in token order (t * top_k + k).  Returns None when the
    operands fall outside the segmented GEMM's contract (the caller then takes
    the unfused path), as the reference's hook does (fused.py:3247-3283).
    """
    if not _DOWN_EPI_ON:
        return None
    if x_rows.dim() != 3 or x_rows.shape[1] != 1:
        return None
    M = order.shape[0]
    if M < MOE_GEMM_MIN_ROWS:
        return None
    if idx_s.dim() != 1 or idx_s.shape[0] != M or row_src.shape != (M,) or w_flat.shape != (M,):
        return None
    up, gate, down = switch_mlp.up_proj, switch_mlp.gate_proj, switch_mlp.down_proj
    parts = [_proj_parts(p) for p in (up, gate, down)]
    if any(p is None for p in parts):
        return None
    (w_up, s_up, b_up), (w_gate, s_gate, b_gate), (w_dn, s_dn, b_dn) = parts
    rows, _, K = x_rows.shape
    x2 = x_rows.reshape(rows, K)
    if not mgg.segmented_eligible(x2, w_up, s_up, b_up, up.group_size, up.bits):
        return None
    H = w_up.shape[1]
    probe = torch.empty((1, H), dtype=x_rows.dtype, device=x_rows.device)
    if not mgg.segmented_eligible(probe, w_dn, s_dn, b_dn, down.group_size, down.bits):
        return None
    top_k = M // rows
    if rows * top_k != M:
        return None
    if _FOLD_MODE == "combine" and w_dn.shape[1] % mc.VEC:
        return None
    _fire.bump(f"moe_fold_block_{_FOLD_MODE}")
    if tables is None:
        counts = mgg.counts_from_sorted_ids(idx_s, w_up.shape[0])
        tables = mgg.segment_tables(counts, bm=MOE_GEMM_BM, mix_threshold=MOE_GEMM_MIX)
    kw = dict(tables=tables, bm=MOE_GEMM_BM, mix_threshold=MOE_GEMM_MIX)
    if _GATHER_FOLD_ON:
        src = row_src
    else:
        src = None
        x2 = x2[row_src.long()]
    x_up = mgg.qmm_segmented(x2, w_up, s_up, b_up, None, row_src=src, group_size=up.group_size, bits=up.bits, **kw)
    x_gate = mgg.qmm_segmented(x2, w_gate, s_gate, b_gate, None, row_src=src, group_size=gate.group_size,
                               bits=gate.bits, **kw)
    act = switch_mlp.activation(x_up, x_gate)
    kw_dn = dict(kw, group_size=down.group_size, bits=down.bits)
    if _FOLD_MODE == "epi":
        # the store writes sorted row s to token row order[s], scaled by its router weight
        scattered = mgg.qmm_segmented(act, w_dn, s_dn, b_dn, None, row_dst=order, row_scale=w_flat[order.long()],
                                      **kw_dn)
        return scattered.reshape(rows, top_k, -1).sum(dim=-2)
    out_sorted = mgg.qmm_segmented(act, w_dn, s_dn, b_dn, None, **kw_dn)
    return mc.combine(out_sorted, inv if inv is not None else inv_perm(order), w_flat, rows, top_k)


def fused_glu_block(switch_mlp, x2: torch.Tensor, idx_flat: torch.Tensor, w_flat: torch.Tensor, top_k: int):
    """sum_k w * down(silu(gate x) * up x).

    Up to ``moe_decode_fused.MAX_PAIRS`` pairs (and shapes its kernel takes):
    one launch, every pair computed on its own.  Otherwise over rows sorted by
    expert, in four launches: the counting sort with the segment tables (one
    route launch up to 16384 rows and 1024 experts, else four), one gathered
    matmul over the fused gate/up bank with the SwiGLU epilogue (x rows read
    through row_src, no gather copy), the down matmul, and the combine (router
    weight, top_k sum).

    x2 (T, K); idx_flat (T*top_k,) expert ids; w_flat (T*top_k,) fp32 router
    weights in token order.  Returns (T, hidden), or None when the block is
    not eligible (other activation, biases, non-affine or mismatched banks,
    or too large for the gathered kernel's tile counters).
    """
    from .nn import swiglu

    if switch_mlp.activation is not swiglu:
        return None
    up, gate, down = switch_mlp.up_proj, switch_mlp.gate_proj, switch_mlp.down_proj
    if any(_proj_parts(p) is None for p in (up, gate, down)):
        return None
    if gate.group_size != up.group_size or gate.bits != up.bits:
        return None
    T = x2.shape[0]
    M = idx_flat.shape[0]
    if M != T * top_k or M == 0:
        return None
    try:
        fw, fs, fb = switch_mlp.fused_gate_up()
    except NotImplementedError:
        return None
    E = up.weight.shape[0]
    if M <= mdf.MAX_PAIRS and down.group_size == gate.group_size and down.bits == gate.bits:
        # decode widths: the whole block in one launch (no sort, no combine)
        y = mdf.glu_block(x2, idx_flat, w_flat, (fw, fs, fb), (down.weight, down.scales, down.biases), top_k,
                          group_size=gate.group_size, bits=gate.bits)
        if y is not None:
            _fire.bump("moe_fused_glu_block")
            return y
    routed = mgg.moe_route(idx_flat, E, top_k)  # sort + tables in one launch for decode / verify batches
    if routed is not None:
        order, idx_s, row_src, inv, tables = routed
    else:
        order, idx_s, row_src, inv, _ = mcs.sort_rows(idx_flat, E, top_k, with_tables=False)
        tables = mgg.gather_tables(idx_s, E)
    try:
        act = mgg.gather_run(x2, fw, fs, fb, tables, row_src=row_src, glu=True, group_size=gate.group_size,
                             bits=gate.bits)
        out = mgg.gather_run(act, down.weight, down.scales, down.biases, tables, group_size=down.group_size,
                             bits=down.bits)
    except NotImplementedError:
        return None
    _fire.bump("moe_fused_glu_block")
    # the down projection above is the stream's previous operation: chained launch
    return mc.combine(out, inv, w_flat, T, top_k, chained=True)


def moe_combine_fold(switch_mlp, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Sparse MoE block output (..., hidden) = sum_k w_k * down(swiglu(gate_k, up_k)).

    ``x`` (..., hidden), ``idx`` (..., top_k) expert ids, ``w`` (..., top_k)
    router weights.  The router weight is applied to the SwiGLU output (cast
    back to x's dtype) before ``down_proj``, as qwen4_exp.py:1796-1805 does.
    """
    top_k = idx.shape[-1]
    lead = idx.shape[:-1]
    hidden = x.shape[-1]
    # the fused block whenever the down-epilogue hook would not take this call
    # (hook off, or fewer rows than its threshold), so both settings agree there
    hook_takes = _DOWN_EPI_ON and idx.numel() >= max(MOE_GEMM_MIN_ROWS, MOE_COMBINE_SORT_MIN)
    if FUSED_GLU and not hook_takes:
        y = fused_glu_block(switch_mlp, x.reshape(-1, hidden), idx.reshape(-1), w.reshape(-1).float(), top_k)
        if y is not None:
            return y.reshape(*lead, -1)
    xx = x.reshape(-1, 1, 1, hidden)  # (rows, 1, 1, hidden)
    do_sort = idx.numel() >= MOE_COMBINE_SORT_MIN
    if do_sort:
        idx_flat = idx.reshape(-1)
        n_experts = switch_mlp.up_proj.weight.shape[0]
        order, idx_s, row_src, inv, tables = mcs.sort_rows(idx_flat, n_experts, top_k, bm=MOE_GEMM_BM,
                                                           mix_threshold=MOE_GEMM_MIX)
        w_flat = w.reshape(-1).float()
        folded = moe_fold_block(switch_mlp, xx.reshape(-1, 1, hidden), row_src, idx_s, order, w_flat,
                                tables=tables, inv=inv)
        if folded is not None:
            return folded.reshape(*lead, -1)
        xs = xx.reshape(-1, 1, hidden)[row_src.long()]
        w_s = w_flat[order.long()][:, None, None]
        idx_u = idx_s
    else:
        xs = xx.expand(*xx.shape[:1], top_k, 1, hidden).reshape(-1, 1, hidden)
        w_s = w.reshape(-1).float()[:, None, None]
        idx_u = idx.reshape(-1)
    x_up = switch_mlp.up_proj(xs, idx_u, sorted_indices=do_sort)
    x_gate = switch_mlp.gate_proj(xs, idx_u, sorted_indices=do_sort)
    act = (switch_mlp.activation(x_up, x_gate).float() * w_s).to(x.dtype)
    out = switch_mlp.down_proj(act, idx_u, sorted_indices=do_sort)  # (M, 1, hidden)
    if do_sort:
        out = out[inv.long()]
    return out.reshape(*lead, top_k, -1).sum(dim=-2)


__all__ = [
    "FUSED_GLU", "MOE_COMBINE_SORT_MIN", "disable_moe_down_epilogue", "enable_moe_down_epilogue",
    "fused_glu_block", "inv_perm", "moe_combine_fold", "moe_fold_block",
]
