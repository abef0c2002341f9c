"""Kernel fire counters (mlxturbo/kernels/_fire.py:1-32).

Host-side counts by name (``bump``/``snapshot``/``reset``, as in the
reference) plus the native library's own per-kernel-family launch counts
(``native``), so a test can tell "slow" from "never ran".
"""

from __future__ import annotations

from collections import Counter

_COUNTS: Counter[str] = Counter()


def bump(name: str, n: int = 1) -> None:
    _COUNTS[name] += n


def snapshot() -> dict[str, int]:
    return dict(_COUNTS)


def reset() -> None:
    _COUNTS.clear()
    from .. import _lib

    _lib.fire_reset()


def native() -> dict[str, int]:
    """Launch counts recorded inside libmlxturbo_b200.so."""
    from .. import _lib

    return _lib.fire_counts()
