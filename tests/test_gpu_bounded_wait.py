"""Failure detection without a GPU fault: a bounded device-side wait that
runs out (an mbarrier nothing completes) returns, raises the library's status
word for the host to read, and leaves the context usable."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from sparsecore_b200 import _native as N

    lib = N.lib()
    st = ctypes.c_uint(0)
    N.check(lib.sl_device_status(1, ctypes.byref(st)))  # clear
    N.check(lib.sl_selftest_bounded_wait(1 << 12, N.stream_ptr(torch.device("cuda", 0))))
    torch.cuda.synchronize()
    N.check(lib.sl_device_status(1, ctypes.byref(st)))  # read and clear
    assert st.value & 1
    N.check(lib.sl_device_status(0, ctypes.byref(st)))
    assert st.value == 0
    # the context is still usable
    a = torch.arange(10.0, device="cuda")
    assert float(a.sum().item()) == 45.0
    assert lib.sl_selftest_bounded_wait(0, None) == N.SL_ERR_INVALID


def test_python_layer_raises_on_timeout():
    """The status check that routers, graph re-captures and the benchmark run
    turns a timed-out wait into RuntimeError, once, and clears the word."""
    from sparsecore_b200 import _native as N

    dev = torch.device("cuda", 0)
    N.check_device_status(dev)  # start clean
    N.check(N.lib().sl_selftest_bounded_wait(1 << 12, N.stream_ptr(dev)))
    with pytest.raises(RuntimeError, match="timed out"):
        N.check_device_status(dev)
    N.check_device_status(dev)  # cleared by the read
