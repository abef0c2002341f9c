"""Route decisions of the dispatch mirror match the reference's router
(mlxturbo/kernels/dispatch.py:102-117, 247-299) row for row.

tests/golden/route_table.json was produced by importing the reference's own
dispatch.py (tests/golden/make_golden.py).  Mirrors bench/test_dispatch_static.py.
"""

import json
import os

import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "route_table.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.fixture()
def dispatch(monkeypatch):
    from mlxturbo_b200.kernels import dispatch as d

    return d


def test_table_rows(golden, dispatch):
    table = {f"{k},{n}": list(row) for (k, n), row in dispatch.DEFAULT_ROUTE_TABLE.items()}
    assert table == golden["table"]


def test_select_route(golden, dispatch):
    for key, routes in golden["select_route_m_-1_to_20"].items():
        k, n = map(int, key.split(","))
        got = [dispatch.select_route(k, n, m) for m in range(-1, 21)]
        assert got == routes, key


@pytest.mark.parametrize("route", ["small_m", "nocap", "mma"])
def test_small_m_rows(golden, dispatch, monkeypatch, route):
    monkeypatch.setenv("MLXTURBO_SMALL_M_ROUTE", route)
    dispatch.refresh_small_m_route()
    for key, row in golden["small_m_rows"][route].items():
        k, n = map(int, key.split(","))
        got = dispatch._small_m_row(k, n)
        assert (None if got is None else list(got)) == row, (route, key)
    monkeypatch.delenv("MLXTURBO_SMALL_M_ROUTE")
    dispatch.refresh_small_m_route()


def test_constants(golden, dispatch):
    assert [dispatch._SMALL_M_MIN, dispatch._SMALL_M_MAX] == golden["small_m_window"]
    assert [dispatch._SMALL_M_N_MIN, dispatch._SMALL_M_K_MIN] == golden["small_m_min_nk"]
    assert dispatch._MMA_M_MIN == golden["mma_m_min"]


def test_bad_env_raises(dispatch, monkeypatch):
    monkeypatch.setenv("MLXTURBO_SMALL_M_ROUTE", "bogus")
    with pytest.raises(ValueError):
        dispatch.refresh_small_m_route()
    monkeypatch.setenv("MLXTURBO_SMALL_M_ROUTE", "off")
    assert dispatch.refresh_small_m_route() is None
    monkeypatch.delenv("MLXTURBO_SMALL_M_ROUTE")
    dispatch.refresh_small_m_route()
    with pytest.raises(ValueError):
        dispatch.select_route(5120, 17408, 6, table={(5120, 17408): ("bogus",) * 17})


def test_enable_swaps_class_in_place(dispatch):
    import torch

    from mlxturbo_b200.nn import QuantizedLinear

    model = torch.nn.Sequential(QuantizedLinear(128, 64), torch.nn.ReLU(), QuantizedLinear(64, 32))
    ids = [id(m) for m in model]
    dispatch.enable(model, active=False)
    assert [id(m) for m in model] == ids
    assert type(model[0]).__name__ == "DispatchedQuantizedLinear"
    assert model[0]._qmm_dispatch_always is False
    dispatch.enable(model)  # idempotent
    assert model[2]._qmm_dispatch_always is True
