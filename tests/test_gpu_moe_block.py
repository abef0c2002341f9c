"""The SparseMoeBlock combine fold and its down-epilogue hook against an fp32
oracle (the reference's gate, bench/test_moe_combine_fold.py: RMS relative
error <= 1e-2 when the fold is on, identical bits below its row threshold)."""

import numpy as np
import pytest
import torch

import oracle as O
from _util import half_to_torch, make_weights, make_x, u32_to_torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _block(rng, E, hidden, inter, gs=64, bits=4):
    from mlxturbo_b200 import nn as qnn

    blk = qnn.SwitchGLU(hidden, inter, E, group_size=gs, bits=bits, device="cuda")
    deq = {}
    for name, (n, k) in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)), ("down_proj", (hidden, inter))):
        ws, ss, bs, ds = [], [], [], []
        for _ in range(E):
            w, s, b = make_weights(rng, n, k, gs, bits)
            ws.append(w)
            ss.append(s)
            bs.append(b)
            ds.append(O.dequantize(w, s, b, k, gs, bits))
        proj = getattr(blk, name)
        proj.weight.copy_(u32_to_torch(np.stack(ws)))
        proj.scales.copy_(half_to_torch(np.stack(ss), "bf16"))
        proj.biases.copy_(half_to_torch(np.stack(bs), "bf16"))
        deq[name] = np.stack(ds)
    return blk, deq


def _oracle(x, idx, w, deq):
    """fp32: sum_k w_k * Wd[e] @ (silu(Wg[e] x) * (Wu[e] x))."""
    xf = x.reshape(-1, x.shape[-1]).astype(np.float32)
    ids = idx.reshape(xf.shape[0], -1)
    wt = w.reshape(xf.shape[0], -1).astype(np.float32)
    out = np.zeros((xf.shape[0], deq["down_proj"].shape[1]), np.float32)
    for t in range(xf.shape[0]):
        for k in range(ids.shape[1]):
            e = ids[t, k]
            g = deq["gate_proj"][e] @ xf[t]
            u = deq["up_proj"][e] @ xf[t]
            a = g / (1.0 + np.exp(-g)) * u
            out[t] += wt[t, k] * (deq["down_proj"][e] @ a)
    return out


def _rms_rel(got, ref):
    return float(np.sqrt(np.mean((got - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-12))


def _inputs(rng, B, S, hidden, E, top_k):
    x = make_x(rng, B * S, hidden).reshape(B, S, hidden)
    idx = np.stack([rng.choice(E, top_k, replace=False) for _ in range(B * S)]).astype(np.int32)
    logits = rng.standard_normal((B * S, E)).astype(np.float32)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    w = np.take_along_axis(p, idx, axis=-1).astype(np.float32)
    return x, idx.reshape(B, S, top_k), w.reshape(B, S, top_k)


def _run(blk, x, idx, w):
    from mlxturbo_b200 import moe

    y = moe.moe_combine_fold(blk, half_to_torch(x, "bf16"), torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


@pytest.mark.parametrize("B,S", [(1, 1), (1, 5), (2, 3), (1, 40)])
def test_unfused_paths(B, S):
    """Below the sort threshold (numel < 64) and above it, fold hook off."""
    from mlxturbo_b200 import moe

    rng = np.random.default_rng(B * 100 + S)
    E, hidden, inter, top_k = 16, 256, 128, 4
    blk, deq = _block(rng, E, hidden, inter)
    x, idx, w = _inputs(rng, B, S, hidden, E, top_k)
    moe.disable_moe_down_epilogue()
    got = _run(blk, x, idx, w)
    ref = _oracle(O.from_half(x), idx, w, deq).reshape(got.shape)
    assert got.shape == (B, S, hidden)
    assert _rms_rel(got, ref) <= TOL


@pytest.mark.parametrize("mode", ["combine", "epi"])
@pytest.mark.parametrize("gather_fold", [True, False])
def test_fold_block(mode, gather_fold):
    """M = rows * top_k >= the GEMM row threshold: gate/up/down through the
    segmented GEMM, then the combine kernel or the scattered store."""
    from mlxturbo_b200 import moe

    rng = np.random.default_rng(17)
    E, hidden, inter, top_k = 16, 256, 128, 8
    blk, deq = _block(rng, E, hidden, inter)
    x, idx, w = _inputs(rng, 2, 64, hidden, E, top_k)  # 128 rows x 8 = 1024
    ref = _oracle(O.from_half(x), idx, w, deq).reshape(2, 64, hidden)
    from mlxturbo_b200.kernels import _fire

    try:
        moe.enable_moe_down_epilogue(mode=mode, gather_fold=gather_fold)
        _fire.reset()
        got = _run(blk, x, idx, w)
        assert _fire.snapshot().get(f"moe_fold_block_{mode}") == 1
    finally:
        moe.disable_moe_down_epilogue()
    assert _rms_rel(got, ref) <= TOL
    unfused = _run(blk, x, idx, w)
    assert _rms_rel(got, unfused) <= TOL


def test_fold_below_threshold_is_unfused_bits():
    """Fewer rows than the GEMM threshold: the hook declines and the result
    has exactly the unfused path's bits."""
    from mlxturbo_b200 import moe

    rng = np.random.default_rng(5)
    E, hidden, inter, top_k = 16, 256, 128, 4
    blk, _ = _block(rng, E, hidden, inter)
    x, idx, w = _inputs(rng, 1, 20, hidden, E, top_k)  # 80 rows
    moe.disable_moe_down_epilogue()
    off = _run(blk, x, idx, w)
    try:
        moe.enable_moe_down_epilogue(mode="combine")
        on = _run(blk, x, idx, w)
    finally:
        moe.disable_moe_down_epilogue()
    assert np.array_equal(on, off)


def test_inv_perm():
    from mlxturbo_b200 import moe

    order = torch.randperm(1000, device="cuda").to(torch.int32)
    assert torch.equal(moe.inv_perm(order).long(), torch.argsort(order.long()))


@pytest.mark.parametrize("B,S", [(1, 1), (1, 5), (2, 20)])
def test_fused_glu_block(B, S):
    """gate/up in one gathered launch with the SwiGLU epilogue, then down and
    the combine: the same block within the reference's fold tolerance."""
    from mlxturbo_b200 import moe
    from mlxturbo_b200.kernels import _fire

    rng = np.random.default_rng(70 + S)
    E, hidden, inter, top_k = 16, 256, 128, 4
    blk, deq = _block(rng, E, hidden, inter)
    x, idx, w = _inputs(rng, B, S, hidden, E, top_k)
    ref = _oracle(O.from_half(x), idx, w, deq).reshape(B, S, hidden)
    _fire.reset()
    got = _run(blk, x, idx, w)
    assert _fire.snapshot().get("moe_fused_glu_block") == 1
    assert _rms_rel(got, ref) <= TOL
    try:
        moe.FUSED_GLU = False  # the projection-by-projection path
        plain = _run(blk, x, idx, w)
    finally:
        moe.FUSED_GLU = True
    assert _rms_rel(plain, ref) <= TOL


def test_gather_run_glu_matches_separate_projections():
    from mlxturbo_b200.kernels import moe_counting_sort as mcs
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    rng = np.random.default_rng(9)
    E, hidden, inter = 8, 256, 192
    blk, _ = _block(rng, E, hidden, inter)
    T = 37
    x = half_to_torch(make_x(rng, T, hidden), "bf16")
    ids = torch.from_numpy(rng.integers(0, E, size=T).astype(np.int32)).cuda()
    order, idx_s, row_src, inv, _ = mcs.sort_rows(ids, E, 1, with_tables=False)
    tables = mgg.gather_tables(idx_s, E)
    fw, fs, fb = blk.fused_gate_up()
    act = mgg.gather_run(x, fw, fs, fb, tables, row_src=row_src, glu=True)
    g = mgg.gather_run(x, blk.gate_proj.weight, blk.gate_proj.scales, blk.gate_proj.biases, tables, row_src=row_src)
    u = mgg.gather_run(x, blk.up_proj.weight, blk.up_proj.scales, blk.up_proj.biases, tables, row_src=row_src)
    ref = torch.nn.functional.silu(g.float()) * u.float()
    torch.cuda.synchronize()
    assert act.shape == (T, inter)
    err = (act.float() - ref).abs().max().item() / max(ref.abs().max().item(), 1.0)
    assert err <= 1e-2, err
