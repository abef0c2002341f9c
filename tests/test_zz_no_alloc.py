"""The allocation-free decode entry point (qmm_quantized_matmul_noalloc).

It exists for callers that cannot allocate device memory while they run --
fixed-arena runtimes, C/FFI hosts without an allocator, serving loops that
may not allocate on a new shape's first call -- and keeps its scratch in an
16 MiB array inside the library.  These tests call it through the C ABI and
compare it with qmm_quantized_matmul (the entry point that takes a caller
workspace) on two calls in a row, including a call of a different shape in
between, since every call shares the built-in array.  This file is collected
last so that a failure here never hides the rest of the suite.
"""

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

import oracle as O
from _util import check_close, half_to_torch, make_weights, make_x, torch_to_half, u32_to_torch

pytestmark = pytest.mark.gpu


def _noalloc(lib, x, w, s, b, M, N, K, gs=64, bits=4, dtype=0):
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    rc = lib.qmm_quantized_matmul_noalloc(x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), y.data_ptr(), M,
                                          N, K, gs, bits, dtype, torch.cuda.current_stream().cuda_stream)
    return rc, y


@pytest.mark.parametrize("N,K,M", [(6144, 5120, 1), (17408, 5120, 4), (5120, 17408, 16), (1032, 2048, 3)])
def test_noalloc_matches_workspace_entry_point(N, K, M):
    from mlxturbo_b200 import _lib, ops

    lib = _lib.load()
    rng = np.random.default_rng(N + K + M)
    w, s, b = make_weights(rng, N, K)
    wt, st, bt = u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16")
    other = make_weights(rng, 777, 1024)
    ow, os_, ob = u32_to_torch(other[0]), half_to_torch(other[1], "bf16"), half_to_torch(other[2], "bf16")
    for call in range(2):
        x = half_to_torch(make_x(rng, M, K), "bf16")
        rc, y = _noalloc(lib, x, wt, st, bt, M, N, K)
        assert rc == _lib.QMM_OK, lib.qmm_last_error()
        ref = ops.quantized_matmul(x, wt, st, bt)
        torch.cuda.synchronize()
        check_close(torch_to_half(y), O.from_half(torch_to_half(ref)), "bf16", f"call {call}")
        assert torch.equal(y, ref), f"call {call}: differs from the workspace entry point"
        # a call of another shape shares the built-in array in between
        rc, _ = _noalloc(lib, half_to_torch(make_x(rng, 2, 1024), "bf16"), ow, os_, ob, 2, 777, 1024)
        assert rc == _lib.QMM_OK, lib.qmm_last_error()
    assert ops.device_error() == 0


def test_noalloc_lm_head_and_bad_shapes():
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda:0")
    x = torch.ones((1, 5120), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((248320, 640), dtype=torch.int32, device=dev)
    s = torch.zeros((248320, 80), dtype=torch.bfloat16, device=dev)
    # the widest decode matrix (the 248320-row lm_head) fits the built-in array:
    # codes 0, scale 0, bias 0 -> every output is 0
    rc, y = _noalloc(lib, x, w, s, s, 1, 248320, 5120)
    assert rc == _lib.QMM_OK, lib.qmm_last_error()
    assert int(torch.count_nonzero(y)) == 0
    rc, _ = _noalloc(lib, torch.zeros((32, 5120), dtype=torch.bfloat16, device=dev), w, s, s, 32, 1024, 5120)
    assert rc == _lib.QMM_EUNSUPPORTED
    del w, s
    torch.cuda.empty_cache()


# The first call on a device looks the built-in array up and clears it on the
# caller's stream; PyTorch side streams are non-blocking, so a clear issued on
# the legacy default stream would not be ordered before that call's kernels.
# A fresh process (this test file may run after others have called the entry
# point) makes its first call from a side stream, on the integer-MMA kernel
# (which keeps an epoch and epoch-tagged partials in the array) and on the
# stream-K kernel, twice each, and compares with the workspace entry point.
_FIRST_CALL_ON_SIDE_STREAM = textwrap.dedent("""
    import sys
    sys.path[:0] = [{repo!r}, {tests!r}, {oracle!r}]
    import numpy as np, torch
    from _util import half_to_torch, make_weights, make_x, u32_to_torch
    from mlxturbo_b200 import _lib, ops
    lib = _lib.load()
    rng = np.random.default_rng(3)
    side = torch.cuda.Stream()
    for N, K, M in ((17408, 5120, 1), (5120, 8192, 3)):
        w, s, b = make_weights(rng, N, K)
        wt, st, bt = u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16")
        for call in range(2):
            x = half_to_torch(make_x(rng, M, K), "bf16")
            torch.cuda.synchronize()
            with torch.cuda.stream(side):
                y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
                rc = lib.qmm_quantized_matmul_noalloc(x.data_ptr(), wt.data_ptr(), st.data_ptr(), bt.data_ptr(),
                                                      y.data_ptr(), M, N, K, 64, 4, 0, side.cuda_stream)
                assert rc == 0, lib.qmm_last_error()
            side.synchronize()
            ref = ops.quantized_matmul(x, wt, st, bt)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), (N, K, M, call)
    assert ops.device_error() == 0
    print("ok")
""")


def test_noalloc_first_call_on_a_side_stream():
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = _FIRST_CALL_ON_SIDE_STREAM.format(repo=repo, tests=os.path.join(repo, "tests"),
                                             oracle=os.path.join(repo, "oracle"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]


def test_noalloc_argument_checks_match_the_workspace_entry_point():
    from mlxturbo_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda:0")
    x = torch.zeros((4, 1024), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((64, 128), dtype=torch.int32, device=dev)
    s = torch.zeros((64, 16), dtype=torch.bfloat16, device=dev)
    y = torch.empty((4, 64), dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    args = (x.data_ptr(), w.data_ptr(), s.data_ptr(), s.data_ptr(), y.data_ptr())
    # M = 0 is a no-op for both entry points
    assert lib.qmm_quantized_matmul_noalloc(*args, 0, 64, 1024, 64, 4, 0, st) == _lib.QMM_OK
    assert lib.qmm_quantized_matmul(*args, 0, 64, 1024, 64, 4, 0, None, 0, st) == _lib.QMM_OK
    # misaligned scales: the same EINVAL, and a fresh message
    bad = (x.data_ptr(), w.data_ptr(), s.data_ptr() + 1, s.data_ptr(), y.data_ptr())
    assert lib.qmm_quantized_matmul_noalloc(*bad, 4, 64, 1024, 64, 4, 0, st) == _lib.QMM_EINVAL
    assert b"aligned" in lib.qmm_last_error()
    assert lib.qmm_quantized_matmul_noalloc(*args, 4, 64, 1024, 64, 4, 0, st) == _lib.QMM_OK
    assert lib.qmm_last_error() == b""
    torch.cuda.synchronize()
