"""Failure detection on the GPU without a fault: a kernel's bounded wait runs out (a barrier phase that nothing
completes), the kernel records it and returns, the host reads JC_ERR_TIMEOUT, and the device stays usable."""

import numpy as np
import pytest

import jitcast_b200
from jitcast_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_device_stays_usable(jc):
    L = _lib.lib()
    assert L.jc_device_wait_selftest(0, 20_000) == _lib.ERR_TIMEOUT  # a 20 ms wait that nothing ends
    assert "gave up" in _lib.last_error()
    assert L.jc_device_sync(0) == _lib.OK  # the error word was read and cleared
    rng = np.random.default_rng(1)
    x = rng.standard_normal((256, 128)).astype(np.float32)
    w = (rng.standard_normal((64, 128)) / 12).astype(np.float32)
    y = jitcast_b200.ops.linear(x, w, None, precision="fp32")
    np.testing.assert_allclose(y, x.astype(np.float64) @ w.T.astype(np.float64), rtol=1e-4, atol=1e-4)
