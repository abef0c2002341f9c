"""Shape-by-M routing for affine quantized linear layers
(mlxturbo/kernels/dispatch.py: route table :14-68, select_route :102-117,
small-M override :247-299, quantized_matmul :302-382, dispatched class and
dispatch_scope :385-466).

The route vocabulary, the measured route table and the small-M override are
kept as data with the reference's exact semantics, so route decisions
(`select_route`, `_small_m_row`) match the reference row for row.  What a route
*runs* differs: every route lands on this package's B200 kernels --

  stock / nocap / small_m / mma / e120 with M <= 16  -> decode kernel (qmv.cu):
      weights streamed once for the whole verify width, so the reference's
      distinction between qmv_fast, qmv_wide (5-row tiles), fast_qmm's MMA
      tile and E120 collapses into one kernel whose rows are bit-identical to
      single-row calls (the property the small_m route was chosen for);
  M > 16 -> tensor-core prefill kernel (prefill.cu).

The route taken is recorded in the fire counters (``_fire``) so the dispatch
decisions stay observable, as in the reference's A/B tooling.  There is no
stock fallback: an unsupported mode or shape raises.
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from contextvars import ContextVar
from math import prod
from typing import Any

from . import _fire

STOCK = "stock"
NOCAP = "nocap"
MMA = "mma"
SMALLM = "small_m"
E120 = "e120"
_ROUTES = frozenset((STOCK, NOCAP, MMA, SMALLM, E120))


def _routes(overrides: dict[int, str] | None = None) -> tuple[str, ...]:
    """An M-indexed route row: M=6..8 MMA, M=9..11 nocap, the rest stock, then overrides."""
    row = [STOCK] * 17
    for m in range(6, 9):
        row[m] = MMA
    for m in range(9, 12):
        row[m] = NOCAP
    if overrides:
        for m, route in overrides.items():
            row[m] = route
    return tuple(row)


def _exact_routes(overrides: dict[int, str]) -> tuple[str, ...]:
    row = [STOCK] * 17
    for m, route in overrides.items():
        row[m] = route
    return tuple(row)


# (K, N) -> route per M (0..16), the reference's measured table.
DEFAULT_ROUTE_TABLE: dict[tuple[int, int], tuple[str, ...]] = {
    (5120, 17408): _routes({5: MMA} | {m: MMA for m in range(9, 17)}),   # MLP up/gate
    (17408, 5120): _routes({m: MMA for m in range(10, 17)}),             # MLP down
    (5120, 12288): _routes({5: MMA} | {m: MMA for m in range(9, 17)}),   # attention q
    (5120, 248320): _routes({5: MMA} | {m: MMA for m in range(9, 17)}),  # lm_head
    (21504, 5376): _exact_routes({4: E120}),
}

_DISPATCHED_CLASS = None
_DISPATCH_ACTIVE = ContextVar("qmm_b200_dispatch_active", default=False)
_E120_ACTIVE = ContextVar("qmm_b200_e120_active", default=True)
_UNLISTED_SMALL_M_ACTIVE = ContextVar("qmm_b200_unlisted_small_m_active", default=True)


def _e120_enabled() -> bool:
    """MLXTURBO_QMM_E120 policy (auto|on|force|off), resolved once per scope.

    On B200 the E120 route runs the same decode kernel, so "auto" enables it.
    """
    mode = os.environ.get("MLXTURBO_QMM_E120", "auto").strip().lower()
    if mode in ("1", "on", "true", "yes", "force", "", "auto"):
        return True
    if mode in ("0", "off", "false", "no", "stock"):
        return False
    raise ValueError("MLXTURBO_QMM_E120 must be auto, on, force, or off")


def select_route(k: int, n: int, m: int, table: dict[tuple[int, int], tuple[str, ...]] | None = None) -> str:
    """Return the route name for one flattened matmul (dispatch.py:102-117)."""
    route_table = DEFAULT_ROUTE_TABLE if table is None else table
    row = route_table.get((k, n))
    if row is None or m < 0 or m >= len(row):
        return STOCK
    route = row[m]
    if route not in _ROUTES:
        raise ValueError(f"invalid quantized-matmul route {route!r}")
    return route


# ----------------------------------------------------------------------------
# small-M override (MLXTURBO_SMALL_M_ROUTE), dispatch.py:247-299
# ----------------------------------------------------------------------------
_SMALL_M_ENV = "MLXTURBO_SMALL_M_ROUTE"
_SMALL_M_MIN = 2
_SMALL_M_MAX = 5
_SMALL_M_N_MIN = 1024
_SMALL_M_K_MIN = 1024
_SMALL_M_ROUTE: str | None = None
_SMALL_M_ROWS: dict[tuple[int, int], tuple[str, ...]] = {}
_MMA_M_MIN = 5


def refresh_small_m_route() -> str | None:
    """Re-read MLXTURBO_SMALL_M_ROUTE (auto|small_m|nocap|mma|off).

    "auto" means small_m: the reference enables it on every non-NAX Apple GPU;
    on B200 the decode kernel is the small_m kernel.
    """
    global _SMALL_M_ROUTE, _SMALL_M_ROWS
    val = os.environ.get(_SMALL_M_ENV, "").strip().lower()
    if val in ("", "auto"):
        val = SMALLM
    elif val in ("0", "off", "stock"):
        val = None
    elif val not in (NOCAP, MMA, SMALLM):
        raise ValueError(f"{_SMALL_M_ENV}={val!r} is unknown (auto / {SMALLM!r} / {NOCAP!r} / {MMA!r} / off)")
    if val != _SMALL_M_ROUTE:
        _SMALL_M_ROUTE = val
        _SMALL_M_ROWS = {}
    return _SMALL_M_ROUTE


def _small_m_row(k: int, n: int) -> tuple[str, ...] | None:
    """The route row with the small-M override applied (None if the shape is too small)."""
    row = _SMALL_M_ROWS.get((k, n))
    if row is not None:
        return row
    if n < _SMALL_M_N_MIN or k < _SMALL_M_K_MIN:
        return None
    base = DEFAULT_ROUTE_TABLE.get((k, n))
    new = list(base) if base is not None else [STOCK] * 17
    for mm in range(_SMALL_M_MIN, _SMALL_M_MAX + 1):
        if new[mm] == STOCK:
            new[mm] = _SMALL_M_ROUTE
    row = tuple(new)
    _SMALL_M_ROWS[(k, n)] = row
    return row


def _route_for(k: int, n: int, m: int, table) -> str:
    route = None
    if (_SMALL_M_ROUTE is not None and table is None and _UNLISTED_SMALL_M_ACTIVE.get()
            and _SMALL_M_MIN <= m <= _SMALL_M_MAX):
        row = _small_m_row(k, n)
        if row is not None:
            route = row[m]
    if route is None:
        route = select_route(k, n, m, table)
    if route == E120 and not _E120_ACTIVE.get():
        route = STOCK
    return route


def quantized_matmul(x, w, scales, biases, *, group_size: int, bits: int, mode: str = "affine",
                     table: dict[tuple[int, int], tuple[str, ...]] | None = None):
    """Dispatch one QuantizedLinear matmul (x [..., K] -> [..., N]) to the B200 kernels."""
    from .. import ops

    if x.dim() < 1:
        raise ValueError("x must have at least one dimension")
    k = x.shape[-1]
    n = w.shape[0]
    m = prod(x.shape[:-1])
    route = _route_for(k, n, m, table)
    _fire.bump(f"route_{route}")
    return ops.quantized_matmul(x, w, scales, biases, transpose=True, group_size=group_size, bits=bits, mode=mode)


# ----------------------------------------------------------------------------
# module patching (dispatch.py:385-466)
# ----------------------------------------------------------------------------

def _get_dispatched_class():
    global _DISPATCHED_CLASS
    if _DISPATCHED_CLASS is None:
        from ..nn import QuantizedLinear

        class DispatchedQuantizedLinear(QuantizedLinear):
            """QuantizedLinear routed by shape-by-M while active."""

            def forward(self, x):
                active = getattr(self, "_qmm_dispatch_always", False) or _DISPATCH_ACTIVE.get()
                if not active:
                    return super().forward(x)
                out = quantized_matmul(x, self.weight, self.scales, self.biases, group_size=self.group_size,
                                       bits=self.bits, mode=self.mode, table=None if active else {})
                if self.bias is not None:
                    out = out + self.bias
                return out

        DispatchedQuantizedLinear.__module__ = __name__
        _DISPATCHED_CLASS = DispatchedQuantizedLinear
    return _DISPATCHED_CLASS


@contextmanager
def dispatch_scope(*, unlisted_small_m: bool = True):
    """Activate verification-only dispatched layers for the duration of the block."""
    refresh_small_m_route()
    active_token = _DISPATCH_ACTIVE.set(True)
    e120_token = _E120_ACTIVE.set(_e120_enabled())
    small_m_token = _UNLISTED_SMALL_M_ACTIVE.set(unlisted_small_m)
    try:
        yield
    finally:
        _UNLISTED_SMALL_M_ACTIVE.reset(small_m_token)
        _E120_ACTIVE.reset(e120_token)
        _DISPATCH_ACTIVE.reset(active_token)


def enable(model: Any, *, active: bool = True):
    """Swap every QuantizedLinear under `model` to the dispatched class in place.

    Changing only ``__class__`` keeps module identity, parameter names and
    loaded tensors; repeated calls are idempotent.  ``active=False`` installs
    verification-only routing for use inside :func:`dispatch_scope`.
    """
    from ..nn import QuantizedLinear

    _E120_ACTIVE.set(_e120_enabled())
    dispatched = _get_dispatched_class()
    for _, module in model.named_modules():
        if isinstance(module, QuantizedLinear) and not isinstance(module, dispatched):
            module.__class__ = dispatched
        if isinstance(module, dispatched):
            module._qmm_dispatch_always = active
    return model


__all__ = [
    "DEFAULT_ROUTE_TABLE", "E120", "MMA", "NOCAP", "SMALLM", "STOCK", "dispatch_scope", "enable",
    "quantized_matmul", "refresh_small_m_route", "select_route",
]
