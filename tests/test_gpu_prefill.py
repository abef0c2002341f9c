"""Parity of the tensor-core prefill kernel (M > 16) against the CPU oracle.

Mirrors bench/test_qmm_wide_shapes.py (shapes (10240,320), (320,10240),
(2560,300) at rows 13..1000; all tile variants bit-identical to each other)
with the fp32 oracle in place of live MLX.  Tolerance: tests/_util.py.
"""

import numpy as np
import pytest
import torch

import oracle as O
from _util import check_close, half_to_torch, make_weights, make_x, torch_to_half, u32_to_torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from mlxturbo_b200 import ops as _ops

    return _ops


def _qmm(ops, x, w, s, b, gs, bits, dtype):
    y = ops.quantized_matmul(half_to_torch(x, dtype), u32_to_torch(w), half_to_torch(s, dtype),
                             half_to_torch(b, dtype), group_size=gs, bits=bits)
    assert ops.device_error() == 0, "a bounded wait inside the prefill kernel gave up"
    return torch_to_half(y)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
def test_prefill_parity_small(ops, bits, gs, dtype):
    rng = np.random.default_rng(bits * 100 + gs)
    M, N, K = 300, 384, 1024
    w, s, b = make_weights(rng, N, K, gs, bits, dtype)
    x = make_x(rng, M, K, dtype)
    check_close(_qmm(ops, x, w, s, b, gs, bits, dtype), O.qmm(x, w, s, b, gs, bits, dtype), dtype,
                f"bits={bits} gs={gs} {dtype}")


@pytest.mark.parametrize("K,N", [(10240, 320), (320, 10240), (2560, 300)])
@pytest.mark.parametrize("M", [17, 32, 100, 250, 1000])
def test_prefill_reference_shapes(ops, K, N, M):
    """The shapes of bench/test_qmm_wide_shapes.py, including N/M tails."""
    rng = np.random.default_rng(K + N + M)
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, M, K, scale=0.1)
    check_close(_qmm(ops, x, w, s, b, 64, 4, "bf16"), O.qmm(x, w, s, b), "bf16", f"{K}->{N} M={M}")


@pytest.mark.parametrize("K", [32, 96, 160, 544])
def test_prefill_k_tails(ops, K):
    """K not a multiple of the 64-wide k-block (group size 32)."""
    rng = np.random.default_rng(K)
    M, N = 70, 200
    w, s, b = make_weights(rng, N, K, 32, 4)
    x = make_x(rng, M, K)
    check_close(_qmm(ops, x, w, s, b, 32, 4, "bf16"), O.qmm(x, w, s, b, 32, 4), "bf16", f"K={K}")


def test_token_tile_does_not_change_bits(ops):
    """128- and 256-token tiles give identical results (the reference's
    all-tiles-bit-identical gate, bench/test_qmm_wide_shapes.py:82-100)."""
    rng = np.random.default_rng(21)
    M, N, K = 520, 256, 2048
    w, s, b = make_weights(rng, N, K)
    xt = half_to_torch(make_x(rng, M, K), "bf16")
    args = (xt, u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"))
    a = ops.prefill_explicit(*args, tokens_per_cta=128)
    c = ops.prefill_explicit(*args, tokens_per_cta=256)
    assert ops.device_error() == 0
    assert torch.equal(a, c)


def test_prefill_rows_independent(ops):
    """A row's result does not depend on the other rows of the call."""
    rng = np.random.default_rng(22)
    M, N, K = 300, 256, 1024
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, M, K)
    full = _qmm(ops, x, w, s, b, 64, 4, "bf16")
    part = _qmm(ops, np.ascontiguousarray(x[37:37 + 150]), w, s, b, 64, 4, "bf16")
    assert np.array_equal(full[37:37 + 150], part)


def test_prefill_production_shape(ops):
    """Prefill qmm of configs[4]: x [512, 5120] against W [17408, 5120] 4-bit g64."""
    rng = np.random.default_rng(23)
    M, N, K = 512, 17408, 5120
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, M, K)
    got = _qmm(ops, x, w, s, b, 64, 4, "bf16")
    rows = np.arange(0, M, 7)  # a strided row sample keeps the oracle fast
    ref = O.qmm(np.ascontiguousarray(x[rows]), w, s, b)
    check_close(got[rows], ref, "bf16", "prefill 512x17408x5120")


def test_prefill_matches_dequantised_reference_exactly_in_products(ops):
    """The prefill kernel multiplies bf16-dequantised weights (as MLX qmm_t
    does): against a float64 matmul of the bf16-rounded dequantised weights the
    only error left is fp32 accumulation and the output rounding."""
    rng = np.random.default_rng(24)
    M, N, K = 128, 128, 512
    w, s, b = make_weights(rng, N, K)
    x = make_x(rng, M, K)
    got = O.from_half(_qmm(ops, x, w, s, b, 64, 4, "bf16")).astype(np.float64)
    deq_bf16 = O.from_half(O.to_half(O.dequantize(w, s, b, K, 64, 4))).astype(np.float64)
    ref = O.from_half(x).astype(np.float64) @ deq_bf16.T
    assert O.normalized_max_error(got, ref) < 4e-3
