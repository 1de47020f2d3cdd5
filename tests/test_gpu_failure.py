"""Failure detection on the GPU without faulting it.

A kernel waits on an mbarrier that nothing arrives on, through the bounded
wait the tcgen05 kernels use; the wait gives up after 50 ms, the device
error word is set, lc_device_status reports LC_ERR_TIMEOUT once, and the
context keeps working (a sum launched afterwards is correct).
"""
import ctypes

import numpy as np
import pytest

from lazy_compiler_b200 import runtime
from oracle import expressions as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_device):
    import torch
    runtime.call("lc_device_status", None)  # clear any earlier state
    runtime.call("lc_selftest_bounded_wait", 50_000_000, None)
    with pytest.raises(runtime.LcError) as err:
        runtime.call("lc_device_status", None)
    assert err.value.status == -4
    assert "code 6" in err.value.message
    runtime.call("lc_device_status", None)  # cleared after being reported
    x = torch.from_numpy(O.uniform(1 << 20, seed=1)).cuda()
    out = torch.empty(1, device="cuda")
    runtime.call("lc_sum_f32", ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), 1 << 20, None)
    assert np.isclose(out.item(), O.sum_(x.cpu().numpy())[0], rtol=1e-5)


def test_selftest_rejects_unbounded_limits(cuda_device):
    for bad in (0, -1, 3_000_000_000):
        with pytest.raises(runtime.LcError) as err:
            runtime.call("lc_selftest_bounded_wait", bad, None)
        assert err.value.status == -1
