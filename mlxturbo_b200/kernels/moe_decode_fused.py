"""The MoE block at decode widths in one launch (C ABI ``qmm_moe_glu_decode``).

The reference's decode MoE (mlxturbo/kernels/moe_decode_fused.py:1-40) runs
the block as per-pair gathered GEMVs with a sort, a SwiGLU op and an unsort
around them, and measured that grouping the pairs of one expert (its
"union read") loses at decode widths; its remaining idea was the per-pair form
without the sort and with gate/up fused (``moe_decode_fused.py:26-32``).
This is that form as one kernel: per (token, expert) pair, gate and up rows
of the interleaved bank with the SwiGLU epilogue, then after one grid barrier
the down rows of every pair of a token summed with the router weights, no
sort and no combine launch.  See ``csrc/moe_decode.cu``.

``glu_block`` returns None when the shapes are outside the kernel, so the
caller can take the four-launch block (``moe.fused_glu_block``).
"""

from __future__ import annotations

import os

import torch

from .. import _lib
from ..ops import _contig, _dtype_code, _stream
from . import _fire

# the largest T * top_k the block takes this kernel for; above it the
# four-launch block, which reads an expert once however many tokens chose it.
# Measured on the 512-expert top-10 block (2048 -> 512 -> 2048, routings
# rotated so the experts come from HBM): T = 1 in 14 us against 31 us; T = 8
# in 61 us against 60 us (80 pair reads against 76 distinct experts).
MAX_PAIRS = int(os.environ.get("MLXTURBO_MOE_DECODE_MAX_PAIRS", "0") or 0) or 20

_WS: dict[int, torch.Tensor] = {}  # per-device workspace: barrier counter + SwiGLU rows


def _workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        size = 1 << 20
        while size < nbytes:
            size <<= 1
        # a new buffer starts at zero (the barrier counter); the old one is
        # released in stream order by the caching allocator
        buf = torch.zeros(size, dtype=torch.uint8, device=dev)
        _WS[idx] = buf
    return buf


def glu_block(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, gate_up: tuple, down: tuple, top_k: int, *,
              group_size: int = 64, bits: int = 4, out: torch.Tensor | None = None) -> torch.Tensor | None:
    """sum_k weights[t,k] * down_e(silu(gate_e x[t]) * up_e x[t]) for x (T, hidden).

    ``ids`` (T * top_k,) or (T, top_k) expert ids, ``weights`` the router
    weights of the same shape (fp32), ``gate_up`` the interleaved bank
    (w [E, 2I, hidden*bits/32], scales, biases) of ``nn.SwitchGLU.fused_gate_up``,
    ``down`` (w [E, hidden, I*bits/32], scales, biases).  Returns (T, hidden),
    or None when the kernel does not take these shapes.
    """
    fw, fs, fb = gate_up
    dw, ds, db = down
    if x.dim() != 2 or not x.is_cuda:
        return None
    T, H = x.shape
    P = ids.numel()
    if P != T * top_k or P == 0 or weights.numel() != P:
        return None
    E, I = dw.shape[0], ds.shape[-1] * group_size
    if fw.shape[0] != E or fw.shape[1] != 2 * I or dw.shape[1] != H:
        return None
    lib = _lib.load()
    dev = x.device
    x = _contig(x)
    ids = _contig(ids.reshape(-1).to(torch.int32))
    weights = _contig(weights.reshape(-1).to(torch.float32))
    fw, fs, fb, dw, ds, db = (_contig(t) for t in (fw, fs, fb, dw, ds, db))
    if out is None:
        out = torch.empty((T, H), dtype=x.dtype, device=dev)
    need = int(lib.qmm_moe_glu_decode_workspace_size(T, top_k, I))
    ws = _workspace(dev, need)
    rc = lib.qmm_moe_glu_decode(x.data_ptr(), ids.data_ptr(), weights.data_ptr(), fw.data_ptr(), fs.data_ptr(),
                                fb.data_ptr(), dw.data_ptr(), ds.data_ptr(), db.data_ptr(), out.data_ptr(), T, top_k,
                                E, H, I, group_size, bits, _dtype_code(x), ws.data_ptr(), ws.numel(), _stream(dev))
    if rc == _lib.QMM_EUNSUPPORTED:
        return None
    _lib.check(rc, "moe_glu_decode")
    _fire.bump("moe_glu_decode")
    return out
