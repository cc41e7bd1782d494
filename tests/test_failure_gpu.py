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


# ---- host-side failure injection (engine options fail_plan_allocs and fail_slot) ----------------------------------
# The reference's PlanCache.run (tornado/PlanCache.java:70-100): a plan that fails to build while other plans are
# cached drops them and is built once more; a second failure propagates with the first attached, and the cache stays
# usable. A multi-GPU forward (one host thread per shard) gathers every shard before it reports, so one failing
# shard neither deadlocks the call nor poisons the engine.

def _timestral():
    from jitcast_b200 import timestral as ts
    from jitcast_b200 import workloads

    c = ts.TimestralConfig(patch_size=16, d_model=128, num_heads=2, mlp_hidden_dim=256, block_schedule=["time"],
                           quantile_knots=ts.default_knots(9), block_size=4, context_length=256).validate()
    w = ts.random_checkpoint(c, seed=3)

    def block(series, seed):
        x, obs, group, _ = workloads.mixed_batch(series, 256, c.patch_size, seed=seed)
        return ts.BlockInput(x, obs, group, 2)

    return ts, c, w, block


def test_plan_allocation_failure_drops_the_cache_and_retries_once(jc):
    ts, c, w, block = _timestral()
    a, b = block(5, 1), block(40, 2)  # two block shapes: two plans
    with ts.TimestralEngine(c, w, precision="fp32") as ref:
        exp_b = ts.B200TimestralForward(ref).predict_block(b)
    with ts.TimestralEngine(c, w, precision="fp32") as eng:
        fwd = ts.B200TimestralForward(eng)
        fwd.predict_block(a)  # a cached plan
        eng.set_option("fail_plan_allocs", 1)  # b's plan fails once: the cache is dropped and the build retried
        got = fwd.predict_block(b)
        np.testing.assert_array_equal(got, exp_b)
        eng.set_option("fail_plan_allocs", 2)  # the retry fails too: out of memory, reported with its shape
        with pytest.raises(jc.JcError, match="out of device memory") as ei:
            fwd.predict_block(a)
        assert ei.value.status == _lib.ERR_OOM
        np.testing.assert_array_equal(fwd.predict_block(b), exp_b)  # the engine is still usable


def test_plan_allocation_failure_with_an_empty_cache_is_reported(jc):
    ts, c, w, block = _timestral()
    with ts.TimestralEngine(c, w, precision="bf16") as eng:
        eng.set_option("fail_plan_allocs", 1)  # nothing cached to drop: no retry
        with pytest.raises(jc.JcError, match="out of device memory") as ei:
            ts.B200TimestralForward(eng).predict_block(block(3, 4))
        assert ei.value.status == _lib.ERR_OOM
        assert np.isfinite(ts.B200TimestralForward(eng).predict_block(block(3, 4))).all()


@pytest.mark.parametrize("ends", ["host", "device"])
def test_a_failing_shard_is_reported_by_slot_without_deadlock(jc, ends):
    ts, c, w, block = _timestral()
    b = block(9, 5)
    with ts.TimestralEngine(c, w, devices=(0,), precision="fp32") as one:
        exp = ts.B200TimestralForward(one, ends=ends).predict_block(b)
    with ts.TimestralEngine(c, w, devices=(0, 0), precision="fp32") as two:  # two slots: two shards on threads
        fwd = ts.B200TimestralForward(two, ends=ends)
        two.set_option("fail_slot", 1)
        with pytest.raises(jc.JcError, match=r"slot 1 \(GPU 0\): injected shard failure") as ei:
            fwd.predict_block(b)
        assert ei.value.status == _lib.ERR_CUDA
        np.testing.assert_allclose(fwd.predict_block(b), exp, rtol=1e-6, atol=1e-6)  # the next call is whole again
        with pytest.raises(jc.JcArgumentError):
            two.set_option("fail_slot", 2)  # no such slot


def test_injection_in_the_other_families(jc):
    from jitcast_b200 import chronos2 as c2
    from jitcast_b200 import tirex2 as tx
    from test_chronos2_gpu import mixed_input, tiny_config as c2_tiny
    from test_tirex2_gpu import univariate_batch
    from test_tirex2_oracle import mixed_batch as tx_batch, tiny_config as tx_tiny

    cc = c2_tiny()
    with c2.Chronos2Engine(cc, c2.random_checkpoint(cc, seed=4), devices=(0, 0), precision="bf16") as eng:
        fwd = c2.B200Chronos2Forward(eng)
        inp = mixed_input(cc, series=9, covariate_groups=2)
        exp = fwd.forward(inp)
        eng.set_option("fail_slot", 0)
        with pytest.raises(jc.JcError, match=r"slot 0 \(GPU 0\)"):
            fwd.forward(inp)
        # a new shape on both slots, every allocation failing (two shards draw from the count on parallel threads,
        # two attempts each): out of memory, and the engine stays usable
        eng.set_option("fail_plan_allocs", 4)
        with pytest.raises(jc.JcError, match="out of device memory"):
            fwd.forward(mixed_input(cc, series=30, covariate_groups=3))
        np.testing.assert_array_equal(fwd.forward(inp), exp)
    tc = tx_tiny()
    with tx.TiRex2Engine(tc, tx.random_checkpoint(tc, seed=11, norm_jitter=0.1), devices=(0, 0),
                         precision="fp16") as eng:
        fwd = tx.B200TiRex2Forward(eng)
        b = tx_batch(tc)
        exp = fwd.forward(b)
        eng.set_option("fail_slot", 1)
        with pytest.raises(jc.JcError, match=r"slot 1 \(GPU 0\)"):
            fwd.forward(b)
        np.testing.assert_array_equal(fwd.forward(b), exp)
        eng.set_option("fail_plan_allocs", 4)  # a new shape, every allocation of both shards failing
        with pytest.raises(jc.JcError, match="out of device memory"):
            fwd.forward(univariate_batch(tc, rows=6, seed=2))
        np.testing.assert_array_equal(fwd.forward(b), exp)
