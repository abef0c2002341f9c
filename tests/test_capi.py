"""The C-ABI library loads on a host without a GPU and exports every entry
point include/mlxturbo_b200.h declares (no compute calls here)."""

import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "mlxturbo_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^QMM_API\s+[\w\s\*]+?\b(qmm_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "qmm_quantized_matmul" in names and "qmm_gather_qmm" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings_without_gpu():
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    assert lib.qmm_status_string(0) == b"QMM_OK"
    assert lib.qmm_status_string(1) == b"QMM_EUNSUPPORTED"
    assert lib.qmm_version() >= 100


def test_argument_validation_needs_no_gpu():
    """Shape/dtype errors are reported before any device work."""
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    rc = lib.qmm_quantized_matmul(None, None, None, None, None, 1, 64, 256, 64, 3, 0, None, 0, None)
    assert rc == _lib.QMM_EUNSUPPORTED and b"bits=3" in lib.qmm_last_error()
    rc = lib.qmm_quantized_matmul(None, None, None, None, None, 1, 64, 250, 64, 4, 0, None, 0, None)
    assert rc == _lib.QMM_EINVAL
    rc = lib.qmm_quantized_matmul(None, None, None, None, None, 1, 64, 256, 64, 4, 7, None, 0, None)
    assert rc == _lib.QMM_EUNSUPPORTED
    rc = lib.qmm_quantized_matmul(None, None, None, None, None, 2, 64, 256, 64, 4, 0, None, 0, None)
    assert rc == _lib.QMM_EINVAL  # null pointers
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.QMM_EUNSUPPORTED, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.QMM_EINVAL, "x")


def test_k_split_independent_of_m():
    """The decode kernel's K split is a function of (N, K) alone."""
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    for N, K in ((6144, 5120), (1024, 5120), (5120, 17408), (248320, 5120)):
        kw = lib.qmm_qmv_k_warps(N, K, 64)
        assert 1 <= kw <= 16


def test_operator_library_loads_first_in_a_fresh_process():
    """The PyTorch operator library, looked up before anything else loaded the
    C ABI library (the first op call of a fresh process), loads and returns."""
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from mlxturbo_b200 import _lib\n"
            "ops = _lib.torch_ops()\n"
            "assert ops is not None and hasattr(ops, 'quantized_matmul_out')\n"
            "print('ok')\n") % repo
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


def test_transfer_pack_and_gather_arguments_need_no_gpu():
    """The transfer helper, the expert-parallel pack and the gathered matmul's
    row stride reject bad arguments before any device work."""
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    assert lib.qmm_copy_kernel(None, None, 0, None) == _lib.QMM_OK  # nothing to copy
    assert lib.qmm_copy_kernel(16, 32, 48, None) == _lib.QMM_EINVAL  # not device-addressable (no GPU, or no mapping)
    assert lib.qmm_copy_kernel(None, None, 32, None) == _lib.QMM_EINVAL
    assert lib.qmm_copy_kernel(16, 32, 24, None) == _lib.QMM_EINVAL  # bytes not a multiple of 16
    assert lib.qmm_copy_kernel(8, 32, 32, None) == _lib.QMM_EINVAL  # dst not 16-byte aligned
    # pack: row_stride must leave room for the id after `hidden` values
    rc = lib.qmm_ep_pack(16, 4, 8, 2, 2, 32, 64, 48, 64, 64, None)
    assert rc == _lib.QMM_EINVAL and b"row_stride" in lib.qmm_last_error()
    rc = lib.qmm_ep_pack(16, -1, 8, 2, 2, 32, 64, 48, 72, 64, None)
    assert rc == _lib.QMM_EINVAL
    # gather: x_stride 0 (K) or a multiple of 8 that is >= K
    rc = lib.qmm_gather_run(16, 16, 16, 16, None, None, None, 16, 8, 8, 100, 4, 64, 256, 64, 4, 0, 0, 16, 1 << 30,
                            None)
    assert rc == _lib.QMM_EINVAL and b"x_stride" in lib.qmm_last_error()
