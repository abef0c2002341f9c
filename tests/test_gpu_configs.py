"""Every configuration the benchmark times, checked against the CPU oracle at
its production size, and the reference-named entry points run on the GPU.

- x [1, 4096] against W [11008, 4096] (4-bit g64), through the
  public op, the shape router (dispatch.quantized_matmul and the dispatched
  layer class, mlxturbo/kernels/dispatch.py:302-423), fast_qmm with its
  layer patch (mlxturbo/fast_qmm.py:334-472) and the allocation-free entry.
- the full 8-bit g64 lm_head, 248320 x 5120, with real quantized
  weights at M = 1, 4 and 16 (the 4-warp-CTA integer-MMA kernel at M <= 8,
  the CTA-per-tile kernel at M = 16), on a strided row sample.
- the MoE block (512 experts, top-10, 2048 -> 512 -> 2048) at
  T = 1, 8, 64, 256 tokens, uniform and Zipf(1.1) routing, through the call
  the benchmark makes, against the fp32 block restricted to the touched
  experts (RMS relative error <= 1e-2, bench/test_moe_combine_fold.py).
- prefill at M = 2048 and 8192 on row samples.
Weights are generated on the device (as the benchmark does) and the codes the
kernels read are copied back for the oracle.  Tolerance: tests/_util.py.
"""

import numpy as np
import pytest
import torch

import oracle as O
from _util import check_close, half_to_torch, torch_to_half, u32_to_torch

pytestmark = pytest.mark.gpu

GS = 64


def _quantized(dev, gen, N, K, bits, slice_rows=32768):
    """N(0, 0.02) weights through the device quantiser, in row slices."""
    from mlxturbo_b200 import ops

    wq = torch.empty((N, K * bits // 32), dtype=torch.int32, device=dev)
    s = torch.empty((N, K // GS), dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(s)
    for r0 in range(0, N, slice_rows):
        r1 = min(N, r0 + slice_rows)
        wq[r0:r1], s[r0:r1], b[r0:r1] = ops.quantize(torch.randn((r1 - r0, K), generator=gen, device=dev) * 0.02,
                                                    GS, bits, dtype=torch.bfloat16)
    return wq, s, b


def _host(wq, s, b, rows=None):
    """Codes, scales and biases of `rows` as the oracle's numpy arrays."""
    if rows is not None:
        idx = torch.as_tensor(rows, device=wq.device)
        wq, s, b = wq[idx], s[idx], b[idx]
    w = wq.cpu().numpy().view(np.uint32)
    return w, torch_to_half(s), torch_to_half(b)


def _row_sample(N, step):
    rows = np.arange(0, N, step)
    return np.unique(np.concatenate([rows, np.arange(N - 40, N)]))  # the last, partial tiles too


# --------------------------------------------------------------------------- configs[0]
def test_config0_single_linear_every_entry_point():
    from mlxturbo_b200 import _lib, fast_qmm, ops
    from mlxturbo_b200 import nn as qnn
    from mlxturbo_b200.kernels import _fire, dispatch

    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    N, K = 11008, 4096
    wq, s, b = _quantized(dev, gen, N, K, 4)
    x = torch.randn((1, K), generator=gen, device=dev).to(torch.bfloat16)
    w_h, s_h, b_h = _host(wq, s, b)
    ref = O.qmm(torch_to_half(x), w_h, s_h, b_h, GS, 4)

    y = ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=4)
    check_close(torch_to_half(y), ref, "bf16", "configs[0] ops.quantized_matmul")

    # the shape router and the dispatched layer (dispatch.py:302-423)
    _fire.reset()
    yd = dispatch.quantized_matmul(x, wq, s, b, group_size=GS, bits=4)
    assert torch.equal(yd, y)
    assert any(k.startswith("route_") for k in _fire.snapshot())
    layer = qnn.QuantizedLinear(K, N, bias=False, group_size=GS, bits=4, device=dev)
    layer.weight.copy_(wq)
    layer.scales.copy_(s)
    layer.biases.copy_(b)
    model = torch.nn.Sequential(layer)
    dispatch.enable(model, active=False)
    assert type(model[0]).__name__ == "DispatchedQuantizedLinear"
    with dispatch.dispatch_scope():
        yl = model(x.reshape(1, 1, K))
    assert yl.shape == (1, 1, N) and torch.equal(yl.reshape(1, N), y)
    assert torch.equal(model(x), y)  # outside the scope: the plain layer forward

    # fast_qmm and its layer patch (fast_qmm.py:334-472)
    yf = fast_qmm.fast_qmm(x, wq, s, b, group_size=GS, bits=4, force_wide=True)
    assert torch.equal(yf, y)
    plain = qnn.QuantizedLinear(K, N, bias=True, group_size=GS, bits=4, device=dev)
    plain.weight.copy_(wq)
    plain.scales.copy_(s)
    plain.biases.copy_(b)
    plain.bias.data.normal_()
    try:
        fast_qmm.enable()
        _fire.reset()
        yp = plain(x)
        assert _fire.snapshot().get("fast_qmm") == 1
    finally:
        fast_qmm.disable()
    assert torch.equal(yp, (y + plain.bias))
    assert torch.equal(plain(x), yp)  # the unpatched forward: same kernel, same bits

    # the allocation-free entry takes the same kernel for this shape
    lib = _lib.load()
    yn = torch.empty_like(y)
    rc = lib.qmm_quantized_matmul_noalloc(x.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(), yn.data_ptr(),
                                          1, N, K, GS, 4, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.QMM_OK, lib.qmm_last_error()
    torch.cuda.synchronize()
    assert torch.equal(yn, y)
    assert ops.device_error() == 0


# --------------------------------------------------------------------------- configs[2]
@pytest.fixture(scope="module")
def lm_head():
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    wq, s, b = _quantized(dev, gen, 248320, 5120, 8)
    yield wq, s, b, gen
    del wq, s, b
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [1, 4, 16])
def test_full_8bit_lm_head(lm_head, M):
    from mlxturbo_b200 import ops

    wq, s, b, gen = lm_head
    N, K = wq.shape[0], 5120
    x = torch.randn((M, K), generator=gen, device=wq.device).to(torch.bfloat16)
    y = ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=8)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    rows = _row_sample(N, 97)
    w_h, s_h, b_h = _host(wq, s, b, rows)
    ref = O.qmm(torch_to_half(x), w_h, s_h, b_h, GS, 8)  # [M, len(rows)]
    got = torch_to_half(y[:, torch.as_tensor(rows, device=y.device)])
    check_close(got, ref, "bf16", f"lm_head 248320x5120 8-bit M={M}")
    # a second call gives the same bits (fixed split-K order)
    assert torch.equal(ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=8), y)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_lm_head_fused_greedy(lm_head, M):
    """Greedy sampling fused with the lm_head (C ABI qmm_quantized_matmul_argmax):
    the logits equal quantized_matmul's bit for bit and the ids are the first
    maximum of those logits.  M <= 8 takes the integer-MMA epilogue, M = 16 the
    second pass over the stored logits; an index offset shifts the ids (a
    column shard)."""
    from mlxturbo_b200 import ops

    wq, s, b, gen = lm_head
    x = torch.randn((M, 5120), generator=gen, device=wq.device).to(torch.bfloat16)
    y, keys = ops.quantized_matmul_argmax(x, wq, s, b, GS, 8)
    ref = ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=8)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    assert torch.equal(ops.argmax_from_keys(keys), torch.argmax(ref.float(), dim=-1))
    _, k2 = ops.quantized_matmul_argmax(x, wq, s, b, GS, 8, index_offset=1000)
    assert torch.equal(ops.argmax_from_keys(k2), torch.argmax(ref.float(), dim=-1) + 1000)
    # ties: the first occurrence wins (all-zero codes, scales and biases: every logit is 0)
    z = torch.zeros_like(wq[:4096])
    zs = torch.zeros_like(s[:4096])
    _, kz = ops.quantized_matmul_argmax(x, z, zs, zs, GS, 8, index_offset=7)
    assert (ops.argmax_from_keys(kz) == 7).all()
    assert ops.device_error() == 0


# --------------------------------------------------------------------------- configs[3]
E, TOPK, HIDDEN, INTER = 512, 10, 2048, 512


@pytest.fixture(scope="module")
def moe_block():
    from mlxturbo_b200 import distributed as D
    from mlxturbo_b200 import nn as qnn
    from mlxturbo_b200 import ops

    dev = torch.device("cuda:0")
    glu = qnn.SwitchGLU(HIDDEN, INTER, E, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(21)
    for proj, (n, k) in ((glu.gate_proj, (INTER, HIDDEN)), (glu.up_proj, (INTER, HIDDEN)),
                         (glu.down_proj, (HIDDEN, INTER))):
        for e0 in range(0, E, 64):
            wq, sc, bi = ops.quantize(torch.randn((64 * n, k), generator=gen, device=dev) * 0.02, GS, 4,
                                      dtype=torch.bfloat16)
            proj.weight[e0:e0 + 64] = wq.view(64, n, -1)
            proj.scales[e0:e0 + 64] = sc.view(64, n, -1)
            proj.biases[e0:e0 + 64] = bi.view(64, n, -1)
    yield D.ExpertParallelSwitchGLU(glu, E, None), glu, gen
    torch.cuda.empty_cache()


def _moe_oracle(glu, x, ids, w):
    """fp32 sum_k w_k * Wd[e] @ (silu(Wg[e] x) * (Wu[e] x)) over the touched experts only."""
    xf = O.from_half(torch_to_half(x)).astype(np.float32)
    out = np.zeros((xf.shape[0], HIDDEN), np.float32)
    for e in np.unique(ids):
        t, k = np.nonzero(ids == e)
        deq = {}
        for name, (n, kk) in (("gate_proj", (INTER, HIDDEN)), ("up_proj", (INTER, HIDDEN)),
                              ("down_proj", (HIDDEN, INTER))):
            p = getattr(glu, name)
            deq[name] = O.dequantize(p.weight[e].cpu().numpy().view(np.uint32), torch_to_half(p.scales[e]),
                                     torch_to_half(p.biases[e]), kk, GS, 4)
        g = xf[t] @ deq["gate_proj"].T
        u = xf[t] @ deq["up_proj"].T
        a = g / (1.0 + np.exp(-g)) * u
        np.add.at(out, t, w[t, k][:, None] * (a @ deq["down_proj"].T))
    return out


@pytest.mark.parametrize("routing", ["uniform", "zipf"])
@pytest.mark.parametrize("T", [1, 8, 64, 256])
def test_moe_block_production_config(moe_block, T, routing):
    from mlxturbo_b200 import ops

    ep, glu, gen = moe_block
    rng = np.random.default_rng(5 + T)
    if routing == "uniform":
        ids = np.stack([rng.choice(E, TOPK, replace=False) for _ in range(T)])
    else:
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        p /= p.sum()
        perm = np.random.default_rng(99).permutation(E)
        ids = np.stack([perm[rng.choice(E, TOPK, replace=False, p=p)] for _ in range(T)])
    dev = glu.gate_proj.weight.device
    idx = torch.from_numpy(ids.astype(np.int32)).to(dev)
    w = torch.softmax(torch.randn((T, TOPK), generator=gen, device=dev), -1)
    x = torch.randn((T, HIDDEN), generator=gen, device=dev).to(torch.bfloat16)
    y = ep(x, idx, w)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = _moe_oracle(glu, x, ids, w.cpu().numpy())
    got = y.float().cpu().numpy()
    rms = float(np.sqrt(np.mean((got - ref) ** 2)) / np.sqrt(np.mean(ref ** 2)))
    assert rms <= 1e-2, f"T={T} {routing}: rms rel {rms:.3e}"
    assert torch.equal(ep(x, idx, w), y)  # deterministic: stable sort, fixed-order sums


# --------------------------------------------------------------------------- configs[4]
@pytest.mark.parametrize("M", [2048, 8192])
def test_prefill_large_m(M):
    from mlxturbo_b200 import ops

    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    N, K = 17408, 5120
    wq, s, b = _quantized(dev, gen, N, K, 4)
    x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
    y = ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=4)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    rows = _row_sample(M, 61)
    ref = O.qmm(torch_to_half(x[torch.as_tensor(rows, device=dev)]), *_host(wq, s, b), GS, 4)
    check_close(torch_to_half(y[torch.as_tensor(rows, device=dev)]), ref, "bf16", f"prefill M={M}")
