"""Host-side contracts of the reference-named kernel modules (no GPU needed):
tile rules and the stock-lane predicate of qmm_wide
(bench/test_qmm_wide_shapes.py:57-72), the skinny MMA's implementation
switches (qmm_skinny_mma.py:224-235) and the layout predicates."""

import pytest
import torch

from mlxturbo_b200.kernels import qmm_skinny_mma as sk
from mlxturbo_b200.kernels import qmm_wide as qw
from mlxturbo_b200.kernels import qmv_small_m as qsm
from mlxturbo_b200.kernels import qmv_wide_nocap as qwn


def test_stock_lane_predicate_boundaries():
    assert not qw.stock_bit_matches(12, 320, 10240)
    assert qw.stock_bit_matches(13, 320, 10240)
    assert not qw.stock_bit_matches(800, 10240, 320)
    assert qw.stock_bit_matches(832, 10240, 320)
    assert not qw.stock_bit_matches(384, 10240, 640)
    assert qw.stock_bit_matches(400, 10240, 640)
    assert not qw.stock_bit_matches(192, 10240, 1280)
    assert qw.stock_bit_matches(193, 10240, 1280)
    assert qw.stock_bit_matches(256, 64, 320)
    assert not qw.stock_bit_matches(256, 128, 320)


@pytest.mark.parametrize("K,N", [(10240, 320), (320, 10240), (2560, 300), (5120, 17408)])
def test_reference_tiles_valid_on_its_shapes(K, N):
    ok = [t for t in qw.TILES.values() if qw.tile_ok(t, K, N) is None]
    assert len(ok) >= 2
    assert qw.tile_ok(qw.STOCK, K, N) is None


def test_tile_rules():
    assert "BK" in qw.tile_ok(qw.Tile(64, 32, 48, 2, 2), 5120, 320)
    assert "K=" in qw.tile_ok(qw.Tile(64, 32, 32, 2, 2), 5136, 320)
    assert "32 KB" in qw.tile_ok(qw.Tile(256, 128, 64, 4, 4), 5120, 320)
    assert qw.Tile(64, 32, 32, 2, 2, xreads=8).name == "m64n32k32w2x2r8"
    assert qw.Tile(64, 32, 32, 2, 2).threads == 128


def test_invalid_tile_raises_before_any_device_work():
    x = torch.zeros(4, 5136, dtype=torch.bfloat16)
    w = torch.zeros(320, 5136 // 8, dtype=torch.int32)
    s = torch.zeros(320, 5136 // 64 + 1, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        qw.qmm_wide(x, w, s, s)


def test_skinny_implementation_switches():
    x = torch.zeros(8, 512, dtype=torch.bfloat16)
    w = torch.zeros(64, 64, dtype=torch.int32)
    s = torch.zeros(64, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        sk.qmm_skinny_mma(x, w, s, s, implementation="v6")
    with pytest.raises(ValueError):
        sk.qmm_skinny_mma(x, w, s, s, use_table=True)


def test_layout_predicates():
    assert sk.eligible_layout(8, 5120, 17408, (17408, 640), (17408, 80), (17408, 80), 64, 4)
    assert not sk.eligible_layout(5, 5120, 17408, (17408, 640), (17408, 80), (17408, 80), 64, 4)
    assert not sk.eligible_layout(8, 5120, 17404, (17404, 640), (17404, 80), (17404, 80), 64, 4)
    assert sk.e120_eligible_layout(4, 5120, 17408, (17408, 640), (17408, 80), (17408, 80), 64, 4)
    assert not sk.e120_eligible_layout(4, 5120 + 64, 17408, (17408, 648), (17408, 81), (17408, 81), 64, 4)
    assert not sk.e120_eligible_layout(10, 5120, 17408, (17408, 640), (17408, 80), (17408, 80), 64, 4)
    # CPU tensors are never eligible for the CUDA kernels
    x = torch.zeros(2, 512, dtype=torch.bfloat16)
    w = torch.zeros(64, 64, dtype=torch.int32)
    s = torch.zeros(64, 8, dtype=torch.bfloat16)
    assert not qsm.eligible(x, w, s, s, 64, 4)
    assert not qwn._eligible(x, w, s, s, 64, 4)
    assert (qsm.M_MIN, qsm.M_MAX, qsm.BLOCK_SIZE) == (1, 8, 512)
    assert (qwn.M_MIN, qwn.M_MAX) == (6, 12)
    assert (sk.M_MIN, sk.M_MAX) == (6, 16)
