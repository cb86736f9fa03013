"""Device-side failure detection, exercised without a fault: a bounded wait
that nothing completes gives up, the host reads SW_ERR_TIMEOUT from the
device error word, and the context keeps working."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from strideweave_b200 import _native as N


def test_probe_limit_is_validated_on_the_host():
    with pytest.raises(ValueError):
        N.check(N.lib.sw_probe_bounded_wait(-1, None))
    with pytest.raises(ValueError):
        N.check(N.lib.sw_probe_bounded_wait(2_000_000_000, None))


@pytest.mark.gpu
def test_a_wait_that_runs_out_reports_a_timeout_and_the_context_stays_usable():
    from strideweave_b200 import kernels
    from tests.gpu_util import empty, to_device, to_host

    status = ctypes.c_int(-1)
    N.check(N.lib.sw_device_status(ctypes.byref(status)))  # start clean
    N.check(N.lib.sw_probe_bounded_wait(20_000_000, None))  # 20 ms on a barrier nothing arrives on
    N.check(N.lib.sw_device_status(ctypes.byref(status)))
    assert status.value == N.SW_ERR_TIMEOUT
    # the word was cleared, and the device still runs kernels correctly
    x = np.random.default_rng(0).standard_normal((64, 256)).astype(np.float32)
    dx, out = to_device(x), empty(64 * 4)
    kernels.reduce_f32("reduce_max", dx.ptr, x.size, 0, [(64, 256)], [(256, 1)], out.ptr)
    np.testing.assert_array_equal(to_host(out, 64, np.float32), x.max(axis=1))
    N.check(N.lib.sw_device_status(ctypes.byref(status)))
    assert status.value == N.SW_OK
    # and the Python side raises the matching exception
    N.check(N.lib.sw_probe_bounded_wait(1_000_000, None))
    with pytest.raises(N.DeviceTimeout):
        N.raise_device_status()
