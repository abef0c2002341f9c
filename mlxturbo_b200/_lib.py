"""ctypes binding of libmlxturbo_b200.so (the C ABI in include/mlxturbo_b200.h).

There is no fallback: if the library is missing or cannot be loaded, importing
an op raises.  Statuses other than QMM_OK become Python exceptions with the
library's own message (QMM_EUNSUPPORTED -> NotImplementedError,
QMM_EINVAL -> ValueError, anything else -> RuntimeError).
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmlxturbo_b200.so")

QMM_OK, QMM_EUNSUPPORTED, QMM_EINVAL, QMM_ECUDA, QMM_ENCCL, QMM_ETIMEOUT = range(6)
QMM_BF16, QMM_F16 = 0, 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/mlxturbo_b200.h
SIGNATURES = {
    "qmm_status_string": (ctypes.c_char_p, [_i]),
    "qmm_last_error": (ctypes.c_char_p, []),
    "qmm_version": (_i, []),
    "qmm_quantized_matmul": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _p, _sz, _p]),
    "qmm_quantized_matmul_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i]),
    "qmm_quantized_matmul_noalloc": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _p]),
    "qmm_quantized_matmul_argmax": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i64, _p, _p, _sz, _p]),
    "qmm_gather_qmm": (_i, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _i, _i, _i, _p, _sz, _p]),
    "qmm_gather_workspace_size": (_sz, [_i64, _i64]),
    "qmm_segmented": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _i, _i, _p, _sz,
                           _p]),
    "qmm_segmented_workspace_size": (_sz, [_i64, _i64]),
    "qmm_segment_tables": (_i, [_p, _i64, _i64, _i, _i, _p, _p, _p, _p]),
    "qmm_segment_tables_from_counts": (_i, [_p, _i64, _i, _i, _p, _p, _p]),
    "qmm_sort_rows": (_i, [_p, _i64, _i64, _i, _p, _p, _p, _p, _p, _sz, _p]),
    "qmm_sort_workspace_size": (_sz, [_i64, _i64]),
    "qmm_moe_combine": (_i, [_p, _p, _p, _p, _i64, _i, _i64, _i, _p]),
    "qmm_moe_combine_rows": (_i, [_p, _i64, _p, _p, _p, _i64, _i, _i64, _i, _p]),
    "qmm_moe_combine_chained": (_i, [_p, _i64, _p, _p, _p, _i64, _i, _i64, _i, _p]),
    "qmm_dequantize": (_i, [_p, _p, _p, _p, _i64, _i64, _i, _i, _i, _p]),
    "qmm_quantize": (_i, [_p, _p, _p, _p, _i64, _i64, _i, _i, _i, _p]),
    "qmm_fire_count": (ctypes.c_longlong, [ctypes.c_char_p]),
    "qmm_fire_names": (ctypes.c_char_p, []),
    "qmm_fire_reset": (None, []),
    "qmm_qmv_explicit": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _p]),
    "qmm_qmv_i8": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _p, _sz, _p]),
    "qmm_qmv_k_warps": (_i, [_i64, _i64, _i]),
    "qmm_prefill_explicit": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _p]),
    "qmm_device_error": (_i, [_i]),
    "qmm_stream_read": (_i, [_p, _sz, _i, _p, _p]),
    "qmm_copy_kernel": (_i, [_p, _p, _sz, _p]),
    "qmm_gather_tables": (_i, [_p, _i64, _i64, _p, _sz, _p]),
    "qmm_moe_route": (_i, [_p, _i64, _i64, _i, _p, _p, _p, _p, _p, _sz, _p]),
    "qmm_ep_pack": (_i, [_p, _i64, _i64, _i64, _i, _p, _i64, _p, _i64, _p, _p]),
    "qmm_moe_glu_decode_workspace_size": (_sz, [_i64, _i64, _i64]),
    "qmm_moe_glu_decode": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _i, _i, _p,
                                _sz, _p]),
    "qmm_gather_run": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i, _i, _i, _i, _p,
                            _sz, _p]),
}

_lib = None
_lock = threading.RLock()  # torch_ops() calls load() while holding it


class QmmError(RuntimeError):
    pass


def load():
    """Load the library once; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is not built; run `python -m mlxturbo_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


TORCH_OPS_PATH = os.path.join(_HERE, "libmlxturbo_b200_torch.so")
_torch_ops = False  # not looked up yet


def _ops_registered(torch) -> bool:
    try:
        torch.ops.mlxturbo_b200.quantized_matmul
    except (AttributeError, RuntimeError):
        return False
    return True


def torch_ops():
    """``torch.ops.mlxturbo_b200`` (the C++ PyTorch operators over the C ABI,
    csrc/torch_ops.cpp) once their library is built, else None."""
    global _torch_ops
    if _torch_ops is False:
        load()
        with _lock:
            if _torch_ops is False:
                ops = None
                if os.path.exists(TORCH_OPS_PATH):
                    import torch

                    load()  # the C ABI library first: the operator library links against it
                    # the build step loads its freshly built copy into this
                    # process; a second registration of the namespace aborts
                    if not _ops_registered(torch):
                        torch.ops.load_library(TORCH_OPS_PATH)
                    ops = torch.ops.mlxturbo_b200
                _torch_ops = ops
    return _torch_ops


def check(rc: int, what: str) -> None:
    if rc == QMM_OK:
        return
    lib = load()
    msg = f"{what}: {lib.qmm_status_string(rc).decode()}: {lib.qmm_last_error().decode()}"
    if rc == QMM_EUNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == QMM_EINVAL:
        raise ValueError(msg)
    raise QmmError(msg)


def fire_counts() -> dict[str, int]:
    lib = load()
    names = lib.qmm_fire_names().decode().split(",")
    return {n: int(lib.qmm_fire_count(n.encode())) for n in names}


def fire_reset() -> None:
    load().qmm_fire_reset()
