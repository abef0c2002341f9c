"""The reference-named kernel entry points on the GPU: each computes
quantized_matmul within the oracle tolerance and keeps its module's
invariant (per-row single-call bits for qmv_small_m, bench/test_qmm_smallm.py:68-84;
all tiles agree for qmm_wide, bench/test_qmm_wide_shapes.py:75-92)."""

import numpy as np
import pytest
import torch

import oracle as O
from _util import check_close, half_to_torch, make_weights, make_x, torch_to_half, u32_to_torch

pytestmark = pytest.mark.gpu


def _args(rng, M, N, K, dtype="bf16"):
    w, s, b = make_weights(rng, N, K, 64, 4, dtype)
    x = make_x(rng, M, K, dtype)
    t = (half_to_torch(x, dtype), u32_to_torch(w), half_to_torch(s, dtype), half_to_torch(b, dtype))
    return t, O.qmm(x, w, s, b, 64, 4, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_qmv_small_m_rows_are_single_row_calls(dtype):
    from mlxturbo_b200.kernels import _fire
    from mlxturbo_b200.kernels import qmv_small_m as qsm

    rng = np.random.default_rng(3)
    (x, w, s, b), ref = _args(rng, 8, 1024, 2048, dtype)
    _fire.reset()
    full = qsm.qmv_small_m(x, w, s, b)
    rows = torch.cat([qsm.qmv_small_m(x[i:i + 1], w, s, b) for i in range(8)])
    assert torch.equal(full, rows)
    assert _fire.snapshot()["qmv_small_m"] == 9
    check_close(torch_to_half(full), ref, dtype, "qmv_small_m")


def test_qmv_wide_nocap():
    from mlxturbo_b200.kernels import qmv_wide_nocap as qwn

    rng = np.random.default_rng(4)
    for M in (6, 9, 12):
        (x, w, s, b), ref = _args(rng, M, 512, 1024)
        check_close(torch_to_half(qwn.qmv_wide_nocap(x, w, s, b)), ref, "bf16", f"qmv_wide_nocap M={M}")


@pytest.mark.parametrize("impl,M", [("v5", 6), ("v5", 16), ("e120_v4", 2), ("e120_v4", 9)])
def test_qmm_skinny_mma(impl, M):
    from mlxturbo_b200.kernels import qmm_skinny_mma as sk

    rng = np.random.default_rng(M)
    (x, w, s, b), ref = _args(rng, M, 1024, 2048)
    got = sk.qmm_skinny_mma(x, w, s, b, implementation=impl)
    check_close(torch_to_half(got), ref, "bf16", f"{impl} M={M}")


@pytest.mark.parametrize("K,N", [(10240, 320), (320, 10240), (2560, 300)])
def test_qmm_wide_all_tiles_agree(K, N):
    from mlxturbo_b200.kernels import qmm_wide as qw

    rng = np.random.default_rng(K + N)
    w, s, b = make_weights(rng, N, K, 64, 4, std=0.05)
    wt, st, bt = u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16")
    probe = torch.zeros(64, K, dtype=torch.bfloat16, device="cuda")
    tiles = [t for t in qw.TILES.values() if qw.eligible(probe, wt, st, bt, t)]
    assert len(tiles) >= 2
    for M in (13, 100, 250):
        xh = make_x(rng, M, K, scale=0.5)
        x = half_to_torch(xh, "bf16")
        outs = [qw.qmm_wide(x, wt, st, bt, tile=t) for t in tiles]
        for t, o in zip(tiles[1:], outs[1:]):
            assert torch.equal(o, outs[0]), f"K={K} N={N} M={M}: {t.name}"
        check_close(torch_to_half(outs[0]), O.qmm(xh, w, s, b), "bf16", f"qmm_wide K={K} N={N} M={M}")


def test_checkpoint_layer_runs_the_kernels(tmp_path):
    """A QuantizedLinear loaded from an MLX-layout safetensors file computes
    quantized_matmul on its tensors as stored (no repacking)."""
    from mlxturbo_b200 import checkpoint as ck

    rng = np.random.default_rng(12)
    w, s, b = make_weights(rng, 512, 1024)
    p = str(tmp_path / "layer.safetensors")
    ck.write_safetensors(p, {"proj.weight": torch.from_numpy(w.view(np.int32)),
                             "proj.scales": half_to_torch(s, "bf16", "cpu"),
                             "proj.biases": half_to_torch(b, "bf16", "cpu")}, u32=["proj.weight"])
    layer = ck.load_quantized_linear(ck.read_safetensors(p, device="cuda"), "proj")
    for M in (1, 4, 40):
        xh = make_x(rng, M, 1024)
        check_close(torch_to_half(layer(half_to_torch(xh, "bf16"))), O.qmm(xh, w, s, b), "bf16", f"M={M}")
