"""Timestral host side on CPU: config parsing, the NumPy mirror of BlockLayout / BlockPrep /
finish against the C oracle's restatement, checkpoint round trip, and engine argument errors."""

import numpy as np
import pytest

from jitcast_b200 import timestral as ts
from jitcast_b200 import workloads
from oracle import timestral as ots


def tiny_config(**kw):
    base = dict(patch_size=16, d_model=128, num_heads=2, mlp_hidden_dim=256,
                block_schedule=["time", "time_variate", "variate_time"], quantile_knots=ts.default_knots(9),
                block_size=4, context_length=512)
    base.update(kw)
    return ts.TimestralConfig(**base).validate()


def block(cfg, series=6, length=256, horizon=2, covariate_groups=2, seed=11):
    x, obs, group, role = workloads.mixed_batch(series, length, cfg.patch_size, seed=seed,
                                                covariate_groups=covariate_groups)
    kf = kfm = None
    if covariate_groups:
        rng = np.random.default_rng(seed + 1)
        kf = rng.standard_normal((x.shape[0], horizon * cfg.patch_size)).astype(np.float32)
        kfm = rng.random((x.shape[0], horizon * cfg.patch_size)) < 0.9
    return ts.BlockInput(x, obs, group, horizon, role if covariate_groups else None, kf, kfm)


def test_config_json_round_trip_and_strict_keys():
    c = ts.config3()
    c2 = ts.TimestralConfig.from_json(c.to_json())
    assert c2 == c
    bad = c.to_json()
    bad["surprise"] = 1
    with pytest.raises(ValueError, match="unknown config key"):
        ts.TimestralConfig.from_json(bad)
    bad = c.to_json()
    bad["mlp_bias"] = True
    with pytest.raises(ValueError, match="not supported"):
        ts.TimestralConfig.from_json(bad)


def test_checkpoint_round_trip(tmp_path):
    c = tiny_config()
    w = ts.random_checkpoint(c, seed=3)
    assert set(w) == set(ts.weight_shapes(c))
    ts.save_checkpoint(tmp_path, c, w)
    c2, w2 = ts.load_checkpoint(tmp_path)
    assert c2 == c
    for k in w:
        np.testing.assert_array_equal(w[k], w2[k])


@pytest.mark.parametrize("covariate_groups", [0, 2])
def test_host_prep_matches_oracle(covariate_groups):
    c = tiny_config()
    b = block(c, covariate_groups=covariate_groups)
    lay = ts.BlockLayout.of(c, b)
    prep = ts.BlockPrep.of(c, lay)
    ref = ots.Model(c, ts.random_checkpoint(c)).prepare(b)
    assert (lay.encoder, lay.horizon, lay.context_patches, int(lay.covariates)) == (
        ref["enc"], ref["horizon"], ref["ll"], ref["covariates"])
    np.testing.assert_array_equal(lay.positions(), ref["positions"])
    np.testing.assert_array_equal(lay.key_valid.astype(np.int32), ref["key_valid"])
    np.testing.assert_array_equal(lay.known.astype(np.int32), ref["known"])
    np.testing.assert_allclose(prep.loc, ref["loc"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(prep.scale, ref["scale"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(prep.tokens, ref["tokens"], rtol=1e-5, atol=1e-6)
    # the same operations in the same order: bit for bit but where NumPy's and the C library's double log differ
    # across a float rounding boundary
    for k in ("tokens", "loc", "scale"):
        assert np.mean(getattr(prep, k) == ref[k]) >= 0.9999, k


def test_host_finish_matches_oracle():
    c = tiny_config()
    b = block(c, covariate_groups=0)
    model = ots.Model(c, ts.random_checkpoint(c))
    out, raw = model.predict_block(b, nthreads=4)
    lay = ts.BlockLayout.of(c, b)
    prep = ts.BlockPrep.of(c, lay)
    mine = prep.finish(c, lay, raw.copy())
    np.testing.assert_allclose(mine, out, rtol=1e-5, atol=1e-5)
    assert np.mean(mine == out) >= 0.9999  # bit for bit but at a rounding boundary of a double transcendental


def test_bucket_sizes():
    # TimestralForward.bucket: x up to 8, then the next multiple of a quarter of its power of two
    assert [ts.bucket(x) for x in (1, 8, 9, 10, 11, 16, 17, 21, 33, 128, 129)] == [1, 8, 10, 10, 12, 16, 20, 24, 40,
                                                                                  128, 160]


def test_context_bucket_pads_in_front_with_empty_patches():
    # TimestralForward.bucketed: a 17-patch context becomes 20 patches, the 3 in front empty. No padded patch is a
    # valid key, the real patches keep their positions and tokens (the scaler's state does not move over unobserved
    # steps), and the oracle's forecasts agree
    c = tiny_config()
    b = block(c, length=17 * c.patch_size)
    p = ts.bucketed_context(b, c.patch_size)
    assert p.inputs.shape[1] == 20 * c.patch_size
    assert ts.bucketed_context(p, c.patch_size) is p
    lay, lp = ts.BlockLayout.of(c, b), ts.BlockLayout.of(c, p)
    assert lp.context_patches == 20 and not lp.key_valid[:, :3].any()
    np.testing.assert_array_equal(lp.key_valid[:, 3:], lay.key_valid)
    np.testing.assert_array_equal(lp.positions()[:, 3:], lay.positions())
    np.testing.assert_array_equal(ts.BlockPrep.of(c, lp).tokens[:, 3:], ts.BlockPrep.of(c, lay).tokens)
    model = ots.Model(c, ts.random_checkpoint(c))
    exact, _ = model.predict_block(b, nthreads=4)
    padded, _ = model.predict_block(p, nthreads=4)
    np.testing.assert_allclose(padded, exact, rtol=1e-5, atol=1e-5)


def test_non_contiguous_series_rejected():
    c = tiny_config()
    b = block(c, covariate_groups=0)
    b.group = np.array([0, 1, 0, 2, 3, 4], np.int32)
    lay = ts.BlockLayout.of(c, b)
    with pytest.raises(ValueError, match="not contiguous"):
        lay.group_ranges()


def test_layout_errors():
    c = tiny_config()
    b = block(c, covariate_groups=0)
    b.horizon_patches = 0
    with pytest.raises(ValueError, match="horizon"):
        ts.BlockLayout.of(c, b)
    b = block(c, covariate_groups=0, length=250)
    with pytest.raises(ValueError, match="multiple of the patch size"):
        ts.BlockLayout.of(c, b)


def test_instance_norm_sums_in_the_reference_order():
    # Scaler.instanceNorm sums in double in its loop order: 1e20 absorbs every 1 that follows it, so the
    # reference's loc is 0 here, where a pairwise sum would keep some of the ones
    x = np.array([1e20] + [1.0] * 15 + [-1e20], np.float32)
    s = 0.0
    for v in x:
        s += float(v)
    loc, _, binary = ts.instance_norm(x, np.ones_like(x, bool), 1e-6)
    assert not binary and loc == np.float32(s / len(x)) == 0.0
