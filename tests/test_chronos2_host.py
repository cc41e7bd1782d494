"""Chronos-2 host side on CPU: config parsing, and the NumPy mirror of ModelLayout / ModelPrep /
finish against the C oracle's restatement on mixed batches (NaN gaps, late starts, groups)."""

import numpy as np
import pytest

from jitcast_b200 import chronos2 as c2
from jitcast_b200 import workloads
from oracle import chronos2 as oc2


def tiny_config(**kw):
    base = dict(d_model=128, d_kv=64, d_ff=256, num_layers=2, num_heads=2, quantiles=[0.1, 0.5, 0.9],
                context_length=256, patch_size=16, max_output_patches=2)
    base.update(kw)
    return c2.Chronos2Config(**base).validate()


def mixed_input(c, series=6, length=300, h=2, covariate_groups=2, seed=11):
    x, obs, group, _ = workloads.mixed_batch(series, length, c.patch_size, seed=seed, covariate_groups=covariate_groups)
    ctx = np.where(obs, x, np.nan).astype(np.float32)
    fut = None
    if covariate_groups:
        rng = np.random.default_rng(seed + 1)
        fut = np.full((x.shape[0], h * c.patch_size - 5), np.nan, np.float32)
        fut[group < covariate_groups] = rng.standard_normal((int((group < covariate_groups).sum()), fut.shape[1]))
    return c2.ModelInput(ctx, group, h, fut)


def test_config_json_round_trip():
    c = c2.config2()
    assert c2.Chronos2Config.from_json(c.to_json()) == c
    bad = c.to_json()
    bad["dense_act_fn"] = "gelu"
    with pytest.raises(ValueError, match="ReLU"):
        c2.Chronos2Config.from_json(bad)


@pytest.mark.parametrize("reg,covariate_groups,length", [(True, 0, 300), (True, 2, 300), (False, 2, 200)])
def test_host_prep_matches_oracle(reg, covariate_groups, length):
    c = tiny_config(use_reg_token=reg)
    inp = mixed_input(c, covariate_groups=covariate_groups, length=length)
    lay = c2.ModelLayout.of(c, inp)
    prep = c2.ModelPrep.of(c, lay)
    ref = oc2.Model(c, c2.random_checkpoint(c)).prepare(inp)
    assert (lay.context_patches, lay.reg, lay.output_patches, lay.tokens) == (ref["nc"], ref["reg"], ref["h"], ref["n"])
    np.testing.assert_array_equal(lay.live.astype(np.int32), ref["live"])
    np.testing.assert_allclose(prep.loc, ref["loc"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(prep.scale, ref["scale"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(prep.tokens, ref["tokens"], rtol=1e-5, atol=1e-6)
    for k in ("tokens", "loc", "scale"):  # bit for bit but at a rounding boundary of a double log
        assert np.mean(getattr(prep, k) == ref[k]) >= 0.9999, k


def test_finish_matches_oracle():
    c = tiny_config()
    inp = mixed_input(c, covariate_groups=0)
    out, raw = oc2.Model(c, c2.random_checkpoint(c)).forward(inp, nthreads=4)
    lay = c2.ModelLayout.of(c, inp)
    prep = c2.ModelPrep.of(c, lay)
    mine = prep.finish(c, lay, raw)
    np.testing.assert_allclose(mine, out, rtol=1e-5, atol=1e-5)
    assert np.mean(mine == out) >= 0.9999  # bit for bit but at a rounding boundary of a double sinh


def test_instance_norm_sums_in_the_reference_order():
    # ModelPrep.instanceNorm sums in double in its loop order: 1e20 absorbs every 1 that follows it (the
    # reference's loc is 0), where a pairwise sum would keep some of them
    c = tiny_config(context_length=16)
    x = np.array([[1e20] + [1.0] * 14 + [-1e20]], np.float32)
    lay = c2.ModelLayout.of(c, c2.ModelInput(x, np.zeros(1, np.int32), 1))
    prep = c2.ModelPrep.of(c, lay)
    s = 0.0
    for v in x[0]:
        s += float(v)
    assert prep.loc[0] == np.float32(s / 16) == 0.0
