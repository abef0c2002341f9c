"""Small-M quantized matmul entry and layer patch (mlxturbo/fast_qmm.py:334-472).

``fast_qmm(x, w, scales, biases, *, group_size, bits, force_wide=False)`` is a
drop-in for ``mx.quantized_matmul(..., transpose=True)``.  On B200 every M in
the reference's window (5..8, and 9..16 with force_wide) and outside it runs
the decode kernel (M <= 16) or the prefill kernel, so ``force_wide`` and the
MLXLM_FAST_QMM_WIDE switch no longer change which kernel runs; they are kept
for call compatibility.  ``enable()``/``disable()`` patch QuantizedLinear's
forward, and the tensor-parallel sharded linears of ``mlxturbo_b200.distributed``
keep their collective step (the reference's TP patch, fast_qmm.py:425-462).
"""

from __future__ import annotations

import os

from . import ops
from .kernels import _fire

M_MIN = 5
M_MAX = 8
M_WIDE_MAX = 16
N_MIN = 4096

_HIST_ON = os.environ.get("MLXLM_QMM_HIST") == "1"
_WIDTH_HIST: dict = {}
_ORIGINAL_FORWARD = None
_ORIGINAL_SHARDED_LOCAL = None


def width_histogram():
    """Call count by M (verification width); diagnostics only (MLXLM_QMM_HIST=1)."""
    return dict(sorted(_WIDTH_HIST.items()))


def fast_qmm(x, w, scales, biases, *, group_size: int, bits: int, force_wide: bool = False):
    K = x.shape[-1]
    M = 1
    for d in x.shape[:-1]:
        M *= d
    if _HIST_ON:
        _WIDTH_HIST[M] = _WIDTH_HIST.get(M, 0) + 1
    _fire.bump("fast_qmm_wide" if M > M_MAX else "fast_qmm")
    del force_wide, K
    return ops.quantized_matmul(x, w, scales, biases, transpose=True, group_size=group_size, bits=bits)


def enable(model=None) -> None:
    """Route QuantizedLinear (and the TP sharded variants) through fast_qmm.

    Patches the class, so layers created later share the path; set
    MLXLM_NO_FAST_QMM=1 to opt out.
    """
    global _ORIGINAL_FORWARD
    from .nn import QuantizedLinear

    if _ORIGINAL_FORWARD is not None or os.environ.get("MLXLM_NO_FAST_QMM") == "1":
        return
    _ORIGINAL_FORWARD = QuantizedLinear.forward

    def forward(self, x):
        if self.mode != "affine":
            return _ORIGINAL_FORWARD(self, x)
        y = fast_qmm(x, self.weight, self.scales, self.biases, group_size=self.group_size, bits=self.bits)
        return y if self.bias is None else y + self.bias

    QuantizedLinear.forward = forward

    # the sharded linears keep their collective (all-gather / all-reduce) and
    # route only the local matmul through fast_qmm (fast_qmm.py:425-462)
    global _ORIGINAL_SHARDED_LOCAL
    from . import distributed as D

    _ORIGINAL_SHARDED_LOCAL = D._ShardedBase._local

    def _local(self, x):
        if self._matmul is not D._qmm:  # a caller-supplied matmul
            return _ORIGINAL_SHARDED_LOCAL(self, x)
        return fast_qmm(x, self.weight, self.scales, self.biases, group_size=self.group_size, bits=self.bits)

    D._ShardedBase._local = _local


def disable() -> None:
    global _ORIGINAL_FORWARD, _ORIGINAL_SHARDED_LOCAL
    from .nn import QuantizedLinear

    if _ORIGINAL_FORWARD is not None:
        QuantizedLinear.forward = _ORIGINAL_FORWARD
        _ORIGINAL_FORWARD = None
    if _ORIGINAL_SHARDED_LOCAL is not None:
        from . import distributed as D

        D._ShardedBase._local = _ORIGINAL_SHARDED_LOCAL
        _ORIGINAL_SHARDED_LOCAL = None
