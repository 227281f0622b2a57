"""Failure detection without a GPU fault: a bounded device-side wait on a
barrier that nothing completes gives up after its limit, reports
FRANK_ETIMEOUT through the device error word, and leaves the context usable
(a normal block call still succeeds afterwards)."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from frank_b200 import _lib, ops

    lib = _lib.load()
    assert ops.read_device_error() == 0
    done = ctypes.c_int32(-1)
    _lib.check(lib.frank_selftest_bounded_wait(50_000_000, ctypes.byref(done),
                                               torch.cuda.current_stream().cuda_stream))
    assert done.value == 0
    assert ops.read_device_error() == _lib.ETIMEOUT
    assert ops.read_device_error() == 0  # reading clears it
    # the context is still healthy
    g = torch.randn(4, 8, device="cuda")
    u = torch.randn(4, 8, device="cuda")
    out = ops.swiglu(g, u)
    ref = g * (u / (1 + torch.exp(-u)))
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-6)


def test_selftest_rejects_bad_limit():
    from frank_b200 import _lib

    lib = _lib.load()
    assert lib.frank_selftest_bounded_wait(0, None, None) == _lib.EINVAL
