"""The MoE block at decode widths in one launch (C ABI qmm_moe_glu_decode,
kernels/moe_decode_fused.py) against the fp32 block oracle, the reference's
fold tolerance (RMS relative error <= 1e-2, bench/test_moe_combine_fold.py),
and against the library's four-launch block; repeated calls and CUDA-graph
replays give identical bits (the grid barrier's counter carries over)."""

import numpy as np
import pytest
import torch

import oracle as O
from _util import half_to_torch, make_weights, make_x, u32_to_torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _block(rng, E, hidden, inter, gs, bits, dtype):
    from mlxturbo_b200 import nn as qnn

    blk = qnn.SwitchGLU(hidden, inter, E, group_size=gs, bits=bits, device="cuda",
                        dtype=torch.float16 if dtype == "f16" else torch.bfloat16)
    deq = {}
    for name, (n, k) in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)), ("down_proj", (hidden, inter))):
        ws, ss, bs, ds = [], [], [], []
        for _ in range(E):
            w, s, b = make_weights(rng, n, k, gs, bits, dtype)
            ws.append(w)
            ss.append(s)
            bs.append(b)
            ds.append(O.dequantize(w, s, b, k, gs, bits, dtype))
        proj = getattr(blk, name)
        proj.weight.copy_(u32_to_torch(np.stack(ws)))
        proj.scales.copy_(half_to_torch(np.stack(ss), dtype))
        proj.biases.copy_(half_to_torch(np.stack(bs), dtype))
        deq[name] = np.stack(ds)
    return blk, deq


def _oracle(xf, ids, wts, deq, E):
    out = np.zeros((xf.shape[0], deq["down_proj"].shape[1]), np.float32)
    for t in range(xf.shape[0]):
        for k in range(ids.shape[1]):
            e = ids[t, k]
            if not 0 <= e < E:
                continue
            g = deq["gate_proj"][e] @ xf[t]
            u = deq["up_proj"][e] @ xf[t]
            out[t] += wts[t, k] * (deq["down_proj"][e] @ (g / (1.0 + np.exp(-g)) * u))
    return out


def _rms_rel(got, ref):
    return float(np.sqrt(np.mean((got - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-12))


def _route(rng, T, E, top_k):
    ids = np.stack([rng.choice(E, top_k, replace=False) for _ in range(T)]).astype(np.int32)
    wts = rng.random((T, top_k)).astype(np.float32)
    return ids, wts / wts.sum(-1, keepdims=True)


def _decode(blk, x, ids, wts, top_k):
    from mlxturbo_b200.kernels import moe_decode_fused as mdf

    d = blk.down_proj
    return mdf.glu_block(x, ids, wts, blk.fused_gate_up(), (d.weight, d.scales, d.biases), top_k,
                         group_size=d.group_size, bits=d.bits)


@pytest.mark.parametrize("E,hidden,inter,top_k,gs,bits,dtype", [
    (8, 512, 256, 4, 32, 4, "bf16"),
    (16, 1024, 512, 8, 64, 4, "bf16"),
    (16, 1024, 512, 8, 64, 4, "f16"),
    (12, 1024, 1024, 3, 128, 4, "bf16"),
    (16, 1024, 512, 8, 64, 8, "bf16"),
    (8, 512, 256, 2, 32, 8, "f16"),
])
@pytest.mark.parametrize("T", [1, 2, 5, 8])
def test_one_launch_block_against_oracle(E, hidden, inter, top_k, gs, bits, dtype, T):
    from mlxturbo_b200 import ops
    from mlxturbo_b200.kernels import _fire

    rng = np.random.default_rng(E * 1000 + hidden + 7 * T + bits + gs)
    blk, deq = _block(rng, E, hidden, inter, gs, bits, dtype)
    x = make_x(rng, T, hidden, dtype)
    ids, wts = _route(rng, T, E, top_k)
    before = _fire.native().get("moe_glu_decode", 0)
    got = _decode(blk, half_to_torch(x, dtype), torch.from_numpy(ids).cuda(), torch.from_numpy(wts).cuda(), top_k)
    assert got is not None
    torch.cuda.synchronize()
    assert _fire.native().get("moe_glu_decode", 0) - before == 1
    ref = _oracle(O.from_half(x, dtype), ids, wts, deq, E)
    assert _rms_rel(got.float().cpu().numpy(), ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("T", [1, 2])
def test_block_dispatch_matches_four_launch_path(T):
    """moe_combine_fold takes the one-launch kernel at decode widths; the
    four-launch block (sort, gathered gate/up, down, combine) agrees."""
    from mlxturbo_b200 import moe
    from mlxturbo_b200.kernels import _fire
    from mlxturbo_b200.kernels import moe_decode_fused as mdf

    rng = np.random.default_rng(300 + T)
    E, hidden, inter, top_k = 32, 1024, 512, 8
    blk, deq = _block(rng, E, hidden, inter, 64, 4, "bf16")
    x = make_x(rng, T, hidden)
    ids, wts = _route(rng, T, E, top_k)
    xt, it, wt = half_to_torch(x, "bf16"), torch.from_numpy(ids).cuda(), torch.from_numpy(wts).cuda()
    before = _fire.native().get("moe_glu_decode", 0)
    one = moe.moe_combine_fold(blk, xt, it, wt).float().cpu().numpy()
    assert _fire.native().get("moe_glu_decode", 0) - before == 1
    saved = mdf.MAX_PAIRS
    try:
        mdf.MAX_PAIRS = 0
        four = moe.moe_combine_fold(blk, xt, it, wt).float().cpu().numpy()
    finally:
        mdf.MAX_PAIRS = saved
    assert _fire.native().get("moe_glu_decode", 0) - before == 1
    ref = _oracle(O.from_half(x), ids, wts, deq, E)
    assert _rms_rel(one, ref) <= TOL
    assert _rms_rel(four, ref) <= TOL
    assert _rms_rel(one, four) <= TOL


def test_repeats_and_graph_replays_are_identical():
    """The grid barrier counts arrivals in windows of the grid size, so calls
    and graph replays follow one another with nothing reset between them."""
    from mlxturbo_b200 import ops

    rng = np.random.default_rng(11)
    E, hidden, inter, top_k, T = 16, 1024, 512, 6, 3
    blk, deq = _block(rng, E, hidden, inter, 64, 4, "bf16")
    x = half_to_torch(make_x(rng, T, hidden), "bf16")
    ids, wts = _route(rng, T, E, top_k)
    it, wt = torch.from_numpy(ids).cuda(), torch.from_numpy(wts).cuda()
    first = _decode(blk, x, it, wt, top_k).clone()
    for _ in range(5):
        assert torch.equal(_decode(blk, x, it, wt, top_k), first)
    out = torch.empty_like(first)
    from mlxturbo_b200.kernels import moe_decode_fused as mdf

    d = blk.down_proj
    fused = blk.fused_gate_up()
    mdf.glu_block(x, it, wt, fused, (d.weight, d.scales, d.biases), top_k, out=out)  # warm-up outside the capture
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        mdf.glu_block(x, it, wt, fused, (d.weight, d.scales, d.biases), top_k, out=out)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(7):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    # eager calls after the replays still line up with the barrier windows
    assert torch.equal(_decode(blk, x, it, wt, top_k), first)
    assert ops.device_error() == 0


def test_ids_outside_the_bank_contribute_nothing():
    from mlxturbo_b200 import ops

    rng = np.random.default_rng(12)
    E, hidden, inter, top_k, T = 8, 512, 256, 4, 3
    blk, deq = _block(rng, E, hidden, inter, 32, 4, "bf16")
    x = make_x(rng, T, hidden)
    ids, wts = _route(rng, T, E, top_k)
    ids[0, 1] = -1
    ids[2, 3] = E + 5
    got = _decode(blk, half_to_torch(x, "bf16"), torch.from_numpy(ids).cuda(), torch.from_numpy(wts).cuda(), top_k)
    ref = _oracle(O.from_half(x), ids, wts, deq, E)
    assert _rms_rel(got.float().cpu().numpy(), ref) <= TOL
    assert ops.device_error() == 0


def test_shapes_outside_the_kernel_decline():
    """inter = 128 is not a multiple of 256: glu_block returns None and the
    MoE block takes the four-launch path."""
    rng = np.random.default_rng(13)
    blk, _ = _block(rng, 8, 256, 128, 64, 4, "bf16")
    x = half_to_torch(make_x(rng, 1, 256), "bf16")
    ids = torch.tensor([[0, 3]], dtype=torch.int32, device="cuda")
    wts = torch.tensor([[0.5, 0.5]], dtype=torch.float32, device="cuda")
    assert _decode(blk, x, ids, wts, 2) is None
