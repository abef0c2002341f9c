"""ops.copy_ / qmm_copy_kernel: pinned host <-> device transfers as one kernel
(the e2e step's activations in and outputs out)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from mlxturbo_b200 import ops as _ops

    return _ops


def test_round_trip_is_exact_and_sees_host_rewrites(ops):
    n = 7 * 5120 + 8
    src = torch.randn(n, dtype=torch.float32).to(torch.bfloat16).pin_memory()
    dev = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    back = torch.empty(n, dtype=torch.bfloat16).pin_memory()
    for rep in range(3):
        src.normal_()  # the host rewrites the buffer between calls: the next copy must see it
        ops.copy_(dev, src)
        ops.copy_(back, dev)
        torch.cuda.synchronize()
        assert torch.equal(back.view(torch.int16), src.view(torch.int16)), rep
        assert torch.equal(dev.cpu().view(torch.int16), src.view(torch.int16)), rep


def test_device_to_device_and_bad_arguments(ops):
    a = torch.randn(4096, device="cuda")
    b = torch.empty_like(a)
    ops.copy_(b, a)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    pageable = torch.empty(4096)
    with pytest.raises(ValueError):
        ops.copy_(pageable, a)  # pageable host memory is not device-addressable
    with pytest.raises(ValueError):
        ops.copy_(b[1:], a[1:])  # not 16-byte aligned
    with pytest.raises(ValueError):
        ops.copy_(b[:10], a)  # sizes differ
