"""The kernels' failure path on the GPU, exercised without a fault: every
mbarrier wait inside the kernels is bounded; when it runs out the kernel
records SFB_ERR_DEVICE_TIMEOUT in the device error word and returns, and the
context stays usable. sfb_selftest_bounded_wait makes such a wait run out
(a barrier that nothing arrives at)."""
import ctypes

import pytest
import torch

from servoflow_b200 import _capi
from servoflow_b200.backend import B200Backend

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(gpu):
    lib = _capi.lib()
    lib.sfb_selftest_bounded_wait.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_int32)]
    lib.sfb_selftest_bounded_wait.restype = ctypes.c_int
    be = B200Backend(0)
    assert be.device_error(reset=True) == 0
    done = ctypes.c_int32(-1)
    _capi.check(lib.sfb_selftest_bounded_wait(2_000_000, ctypes.byref(done)), "self-test")   # 2 ms
    assert done.value == 0                                  # the wait gave up
    assert be.device_error(reset=True) == _capi.SFB_ERR_DEVICE_TIMEOUT
    assert be.device_error(reset=True) == 0                 # the word was reset
    # out-of-range limits are refused, not launched
    assert lib.sfb_selftest_bounded_wait(10, ctypes.byref(done)) == _capi.SFB_ERR_INVALID
    # the context is still usable: a normal attention call works
    q = torch.randn(1, 4, 67, 64, device=gpu).bfloat16()
    out = torch.empty_like(q)
    be.attention(q, q, q, out)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert be.device_error(reset=True) == 0
