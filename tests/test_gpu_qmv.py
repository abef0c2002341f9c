"""Parity of the decode / verify kernel (M <= 16) against the CPU oracle.

Mirrors the reference's numerical gates (bench/test_qmm_smallm.py,
bench/test_dispatch.py, bench/test_qmv_wide_nocap.py) with the oracle in place
of live stock MLX.  Tolerance: tests/_util.py check_close.
"""

import numpy as np
import pytest
import torch

import oracle as O
from _util import check_close, half_to_torch, make_random_codes, make_weights, make_x, torch_to_half, u32_to_torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from mlxturbo_b200 import ops as _ops

    return _ops


def _run(ops, x, w, s, b, gs, bits, dtype):
    y = ops.quantized_matmul(half_to_torch(x, dtype), u32_to_torch(w), half_to_torch(s, dtype),
                             half_to_torch(b, dtype), group_size=gs, bits=bits)
    torch.cuda.synchronize()
    return torch_to_half(y)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 16])
def test_qmv_parity_small(ops, M, bits, gs, dtype):
    rng = np.random.default_rng(1000 * M + 10 * bits + gs)
    N, K = 200, 1024
    w, s, b = make_weights(rng, N, K, gs, bits, dtype)
    x = make_x(rng, M, K, dtype)
    got = _run(ops, x, w, s, b, gs, bits, dtype)
    ref = O.qmm(x, w, s, b, gs, bits, dtype)
    check_close(got, ref, dtype, f"M={M} bits={bits} gs={gs} {dtype}")


@pytest.mark.parametrize("bits,gs,dtype", [(4, 64, "bf16"), (4, 64, "f16"), (4, 32, "bf16"), (4, 128, "f16"),
                                            (8, 64, "bf16"), (8, 32, "f16"), (8, 128, "bf16")])
@pytest.mark.parametrize("M", [1, 3, 4, 5, 8])
def test_integer_mma_decode(ops, M, bits, gs, dtype):
    """The integer-MMA decode kernel (C ABI qmm_qmv_i8) against the oracle on
    small shapes (the dispatcher sends it matrices of 12 MiB and more): few
    units, N tails inside a 32-row tile, tiles cut across warps; rows of an
    M-row call have the bits of single-row calls."""
    from mlxturbo_b200.kernels import _fire

    rng = np.random.default_rng(131 * M + 5 * bits + gs)
    for N, K in ((1, 1024), (129, 1024), (300, 2048), (40, 8192)):
        w, s, b = make_weights(rng, N, K, gs, bits, dtype)
        x = make_x(rng, M, K, dtype)
        args = (half_to_torch(x, dtype), u32_to_torch(w), half_to_torch(s, dtype), half_to_torch(b, dtype))
        if not (K % (1024 // bits) == 0 and (K // gs) % 8 == 0):
            with pytest.raises(NotImplementedError):
                ops.qmv_i8(*args, group_size=gs, bits=bits)
            continue
        before = _fire.native().get("qmv_i8", 0)
        got = ops.qmv_i8(*args, group_size=gs, bits=bits)
        assert _fire.native().get("qmv_i8", 0) - before == 1
        check_close(torch_to_half(got), O.qmm(x, w, s, b, gs, bits, dtype), dtype,
                    f"i8 N={N} K={K} M={M} bits={bits} gs={gs} {dtype}")
        if M > 1:
            single = torch.cat([ops.qmv_i8(args[0][m:m + 1], *args[1:], group_size=gs, bits=bits) for m in range(M)])
            assert torch.equal(got, single), f"rows of the M={M} call differ from single-row calls"
    assert ops.device_error() == 0


def test_integer_mma_decode_graph_replays(ops):
    """Split tiles are summed from partials tagged with a per-call epoch that
    the prep kernel advances on the device: replays of one captured call (same
    workspace, same arguments) with new activations each give that replay's
    result, never a stale partial from the replay before."""
    rng = np.random.default_rng(2027)
    N, K = 4096, 5120  # 128 row tiles x 20 stages over up to 2368 warps: every tile is split
    w, s, b = make_weights(rng, N, K)
    wt, st, bt = u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16")
    x = torch.empty((1, K), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((1, N), dtype=torch.bfloat16, device="cuda")
    xs = [make_x(rng, 1, K) for _ in range(4)]
    x.copy_(half_to_torch(xs[0], "bf16"))
    ops.qmv_i8(x, wt, st, bt, out=y)  # workspace and launch set-up before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.qmv_i8(x, wt, st, bt, out=y)
    for r in range(1, 4):
        x.copy_(half_to_torch(xs[r], "bf16"))
        g.replay()
        torch.cuda.synchronize()
        check_close(torch_to_half(y), O.qmm(xs[r], w, s, b, 64, 4), "bf16", f"replay {r}")
        eager = ops.qmv_i8(x, wt, st, bt)
        assert torch.equal(y, eager), f"replay {r} differs from an eager call"
    del g
    assert ops.device_error() == 0


@pytest.mark.parametrize("N,K,bits", [(17408, 5120, 4), (5120, 5120, 8)])
def test_wide_verify_on_large_matrices(ops, N, K, bits):
    """M = 9..16 on matrices of >= 24 MiB with K = 5120 take the CTA-per-tile
    kernel (32-row tiles, 4 K-warps): parity with the oracle, and rows of an
    M = 9 call equal the first rows of the M = 16 call (one schedule)."""
    rng = np.random.default_rng(N + K + bits)
    w, s, b = make_weights(rng, N, K, 64, bits)
    x = make_x(rng, 16, K)
    wide = _run(ops, x, w, s, b, 64, bits, "bf16")
    check_close(wide, O.qmm(x, w, s, b, 64, bits), "bf16", f"N={N} K={K} bits={bits} M=16")
    assert np.array_equal(_run(ops, x[:9], w, s, b, 64, bits, "bf16"), wide[:9]), "M=9 rows differ from M=16"
    assert ops.device_error() == 0


def test_dispatch_takes_integer_kernel_for_large_matrices(ops):
    """qmm_quantized_matmul sends M <= 8 calls on a >= 12 MiB matrix to the
    integer-MMA kernel and smaller matrices to the warp-MMA kernels."""
    from mlxturbo_b200.kernels import _fire

    rng = np.random.default_rng(77)
    big = make_weights(rng, 17408, 5120)
    mid = make_weights(rng, 5120, 6144)  # 15 MiB
    small = make_weights(rng, 1024, 5120)
    for (w, s, b), want in ((big, 1), (mid, 1), (small, 0)):
        x = make_x(rng, 2, w.shape[1] * 8)  # K from the packed 4-bit rows
        before = _fire.native().get("qmv_i8", 0)
        got = _run(ops, x, w, s, b, 64, 4, "bf16")
        assert _fire.native().get("qmv_i8", 0) - before == want
        check_close(got, O.qmm(x, w, s, b), "bf16", f"dispatch N={w.shape[0]}")


@pytest.mark.parametrize("M", [1, 4, 7, 16])
def test_qmv_random_codes(ops, M):
    """Random uint32 codes + uniform scales/biases, as the reference's gates draw them."""
    rng = np.random.default_rng(M)
    N, K = 1024, 1024
    w, s, b = make_random_codes(rng, N, K)
    x = make_x(rng, M, K, scale=0.05)
    got = _run(ops, x, w, s, b, 64, 4, "bf16")
    check_close(got, O.qmm(x, w, s, b, 64, 4, "bf16"), "bf16", f"random codes M={M}")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_rows_bit_match_single_row_calls(ops, dtype):
    """Each row of an M-row call (M <= 8) has the bits of the M=1 call
    (bench/test_qmm_smallm.py:68-84, the qmv_small_m guarantee)."""
    rng = np.random.default_rng(7)
    N, K = 1032, 2048
    w, s, b = make_weights(rng, N, K, 64, 4, dtype)
    x = make_x(rng, 16, K, dtype)
    single = np.concatenate([_run(ops, x[v:v + 1], w, s, b, 64, 4, dtype) for v in range(16)])
    for M in (2, 3, 4, 5, 8):
        got = _run(ops, x[:M], w, s, b, 64, 4, dtype)
        assert np.array_equal(got, single[:M]), f"M={M}: rows differ from single-row calls"
    # M = 9..16 (the reference's MMA window, which is not bit-identical to M=1
    # either, dispatch.py:232-236) share one schedule among themselves.
    wide = _run(ops, x[:16], w, s, b, 64, 4, dtype)
    for M in (9, 12):
        assert np.array_equal(_run(ops, x[:M], w, s, b, 64, 4, dtype), wide[:M]), f"M={M}"
    check_close(wide, O.qmm(x[:16], w, s, b, 64, 4, dtype), dtype, "M=16")


def test_tile_shape_does_not_change_bits(ops):
    """rows-per-warp changes which warp owns a row, never the reduction order
    (the reference's all-tiles-bit-identical gate, bench/test_qmm_wide_shapes.py:82-100)."""
    rng = np.random.default_rng(11)
    N, K = 777, 2048
    w, s, b = make_weights(rng, N, K)
    x = half_to_torch(make_x(rng, 6, K), "bf16")
    args = (x, u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"))
    for kw in (1, 3, 8):
        a = ops.qmv_explicit(*args, rows_per_warp=1, k_warps=kw)
        c = ops.qmv_explicit(*args, rows_per_warp=2, k_warps=kw)
        assert torch.equal(a, c), f"k_warps={kw}"
        check_close(torch_to_half(a), O.qmm(torch_to_half(x), w, s, b), "bf16", f"k_warps={kw}")


@pytest.mark.parametrize("N,K", [(6144, 5120), (1024, 5120), (5120, 6144), (17408, 5120), (5120, 17408)])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_qmv_production_shapes(ops, N, K, M):
    """The 27B-class decoder shapes of the decode/verify benchmark."""
    rng = np.random.default_rng(N + K + M)
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, M, K)
    got = _run(ops, x, w, s, b, 64, 4, "bf16")
    check_close(got, O.qmm(x, w, s, b), "bf16", f"{N}x{K} M={M}")


@pytest.mark.parametrize("N", [1, 7, 16, 17, 33, 100])
def test_qmv_n_edges(ops, N):
    rng = np.random.default_rng(N)
    K = 512
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, 3, K)
    check_close(_run(ops, x, w, s, b, 64, 4, "bf16"), O.qmm(x, w, s, b), "bf16", f"N={N}")


@pytest.mark.parametrize("K", [64, 128, 192, 640])
def test_qmv_k_tails(ops, K):
    """K not a multiple of 512 (e.g. the MoE down projection's K=640, moe_verify_gather.py:149-166)."""
    rng = np.random.default_rng(K)
    N = 96
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, 5, K)
    check_close(_run(ops, x, w, s, b, 64, 4, "bf16"), O.qmm(x, w, s, b), "bf16", f"K={K}")


def test_lm_head_8bit_slice(ops):
    """8-bit g64 lm_head rows; a column slice keeps the oracle fast."""
    rng = np.random.default_rng(5)
    N, K = 4096, 5120
    w, s, b = make_weights(rng, N, K, 64, 8)
    for M in (1, 5, 16):
        x = make_x(rng, M, K)
        check_close(_run(ops, x, w, s, b, 64, 8, "bf16"), O.qmm(x, w, s, b, 64, 8), "bf16", f"8-bit M={M}")


def test_leading_dims_and_out(ops):
    rng = np.random.default_rng(3)
    N, K = 256, 512
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, 6, K)
    xt = half_to_torch(x, "bf16").reshape(2, 3, K)
    y = ops.quantized_matmul(xt, u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"))
    assert y.shape == (2, 3, N)
    check_close(torch_to_half(y.reshape(6, N)), O.qmm(x, w, s, b), "bf16", "3-D x")


def test_errors_are_loud(ops):
    rng = np.random.default_rng(0)
    w, s, b = make_weights(rng, 64, 256)
    x = half_to_torch(make_x(rng, 2, 256), "bf16")
    wt, st, bt = u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16")
    with pytest.raises(NotImplementedError):
        ops.quantized_matmul(x.float(), wt, st.float(), bt.float())
    with pytest.raises(NotImplementedError):
        ops.quantized_matmul(x, wt, st, bt, mode="mxfp4")
    with pytest.raises(ValueError):
        ops.quantized_matmul(x, wt, st, bt, bits=8)
    with pytest.raises(ValueError):
        ops.quantized_matmul(x.cpu(), wt, st, bt)
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    rc = lib.qmm_quantized_matmul(x.data_ptr(), wt.data_ptr(), st.data_ptr(), bt.data_ptr(), x.data_ptr(), 2, 64,
                                  256, 64, 3, 0, None, 0, None)
    assert rc == _lib.QMM_EUNSUPPORTED and b"bits=3" in lib.qmm_last_error()


@pytest.mark.parametrize("N,K", [(96, 1024), (1024, 5120), (5120, 17408), (700, 4096)])
def test_stream_k_repeatable(ops, N, K):
    """Tiles split across warps are summed through the workspace in a fixed
    order and the tile counters reset themselves: repeated calls (and calls
    with other shapes in between) give identical bits."""
    rng = np.random.default_rng(N * 3 + K)
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, 4, K)
    first = _run(ops, x, w, s, b, 64, 4, "bf16")
    check_close(first, O.qmm(x, w, s, b), "bf16", f"{N}x{K}")
    w2, s2, b2 = make_weights(rng, 333, 1024)
    for _ in range(3):
        _run(ops, make_x(rng, 2, 1024), w2, s2, b2, 64, 4, "bf16")
        assert np.array_equal(_run(ops, x, w, s, b, 64, 4, "bf16"), first)
    assert ops.device_error() == 0


def test_workspace_shared_across_shapes(ops):
    """One workspace serves calls of different shapes: a small matrix's
    partial sums never land on a larger matrix's tile counters."""
    rng = np.random.default_rng(31)
    big = make_weights(rng, 1032, 2048)
    xb = make_x(rng, 2, 2048)
    fresh = _run(ops, xb, *big, 64, 4, "bf16")
    for n, k in ((200, 1024), (96, 512), (4100, 1024), (200, 4096)):
        w, s, b = make_weights(rng, n, k)
        _run(ops, make_x(rng, 3, k), w, s, b, 64, 4, "bf16")
    assert np.array_equal(_run(ops, xb, *big, 64, 4, "bf16"), fresh)
    check_close(fresh, O.qmm(xb, *big), "bf16", "shared workspace")
