"""The Chronos-2 forward on a B200 through the C ABI, against the C restatement of the reference's
FP32 CPU forward (CpuChronos2.forward) on the same seeded inputs and random-init weights.

Inputs follow the reference's batch-parity test (Chronos2BatchParityAccelTest.java:45-114: random walks
plus a daily sinusoid, NaN gaps, late starts, multi-row groups with known future covariates); the
error is max|a − e| / max|e| on every quantile level. Bars (parity_bars): FP32 (the FP32-accumulate mode)
1e-4 on the tiny model (the reference's FP32 device bar) and the north star's 1e-3 on config 2; TF32 1e-3, BF16
and FP16 1e-2, or 2 × the error of the oracle run with its GEMM operands rounded to the mode's format where
that is larger (the reference's rule for reduced-precision device paths).
"""

import numpy as np
import pytest

from jitcast_b200 import chronos2 as c2
from jitcast_b200 import workloads
from oracle import chronos2 as oc2
import parity_bars as pb

pytestmark = pytest.mark.gpu



def per_quantile_err(actual, expected):
    """Out is [rows, Q, h·P]: the error of each quantile level relative to that level's largest value."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert not np.isnan(a).any()
    return max(np.abs(a[:, k] - e[:, k]).max() / max(np.abs(e[:, k]).max(), 1e-6) for k in range(e.shape[1]))


def tiny_config(**kw):
    base = dict(d_model=128, d_kv=64, d_ff=256, num_layers=2, num_heads=2, quantiles=[0.1, 0.5, 0.9],
                context_length=256, patch_size=16, max_output_patches=2)
    base.update(kw)
    return c2.Chronos2Config(**base).validate()


def mixed_input(c, series=7, length=300, h=2, covariate_groups=2, seed=11, shuffle=False):
    x, obs, group, _ = workloads.mixed_batch(series, length, c.patch_size, seed=seed, covariate_groups=covariate_groups)
    ctx = np.where(obs, x, np.nan).astype(np.float32)
    fut = None
    if covariate_groups:
        rng = np.random.default_rng(seed + 1)
        fut = np.full((x.shape[0], h * c.patch_size - 3), np.nan, np.float32)
        sel = group < covariate_groups
        fut[sel] = rng.standard_normal((int(sel.sum()), fut.shape[1]))
    if shuffle:  # rows of a group need not be adjacent in the caller's order
        perm = np.random.default_rng(seed + 2).permutation(len(group))
        ctx, group = ctx[perm], group[perm]
        fut = None if fut is None else fut[perm]
    return c2.ModelInput(ctx, group, h, fut)


@pytest.fixture(scope="module")
def tiny():
    c = tiny_config()
    w = c2.random_checkpoint(c, seed=4)
    return c, w, oc2.Model(c, w)


@pytest.mark.parametrize("precision", ["fp32", "tf32", "bf16", "fp16"])
@pytest.mark.parametrize("covariate_groups,shuffle", [(0, False), (2, True)])
def test_tiny_model_matches_oracle(jc, tiny, precision, covariate_groups, shuffle):
    c, w, model = tiny
    inp = mixed_input(c, covariate_groups=covariate_groups, shuffle=shuffle)
    exp, _ = model.forward(inp)
    bar, floor = pb.bar(precision, lambda: model.forward(inp)[0], lambda o: per_quantile_err(o, exp), pb.TINY)
    with c2.Chronos2Engine(c, w, precision=precision) as eng:
        fwd = c2.B200Chronos2Forward(eng)  # the host ends on the GPU (the default)
        got = fwd.forward(inp)
        got2 = fwd.forward(inp)  # graph replay
        got_host = c2.B200Chronos2Forward(eng, ends="host").forward(inp)  # jc_forward_chronos2
    assert got.shape == exp.shape
    err = per_quantile_err(got, exp)
    print(f"tiny {precision}: per-quantile rel max err {err:.3e} (bar {bar:.3e}, floor {floor})")
    assert err < bar, f"{precision}: per-quantile rel max err {err:.3e} (bar {bar:.3e})"
    err_host = per_quantile_err(got_host, exp)
    assert err_host < bar, f"{precision}, host ends: per-quantile rel max err {err_host:.3e} (bar {bar:.3e})"
    np.testing.assert_array_equal(got, got2)


def ends_input(c, case):
    inp = mixed_input(c, covariate_groups=0 if case == "plain" else 2, shuffle=case == "covariates")
    if case == "degenerate":
        ctx = inp.context.copy()
        ctx[0] = np.where(np.isnan(ctx[0]), np.nan, np.float32(3.0))  # constant: InstanceNorm's scale floor 1e-5
        ctx[1] = np.nan  # nothing observed: (loc, scale) = (0, 1)
        inp = c2.ModelInput(ctx, inp.group, inp.output_patches, inp.future_covariates)
    return inp


@pytest.mark.parametrize("case", ["plain", "covariates", "degenerate"])
@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_host_ends_on_device_match_host_ends(jc, tiny, case, precision):
    # ModelPrep.of and ModelPrep.finish on the GPU (jc_forecast_chronos2) against the same engine with both ends
    # on the host: the reference's arithmetic operation for operation, so equal bit for bit except where a double
    # log or sinh (CUDA's against NumPy's) lands within an ulp of a float rounding boundary; both meet the bar
    c, w, model = tiny
    inp = ends_input(c, case)
    exp, _ = model.forward(inp)
    with c2.Chronos2Engine(c, w, precision=precision) as eng:
        host = c2.B200Chronos2Forward(eng, ends="host").forward(inp)
        fwd = c2.B200Chronos2Forward(eng, ends="device")
        dev = fwd.forward(inp)
        dev2 = fwd.forward(inp)  # graph replay, staged buffers reused
    assert dev.shape == host.shape == exp.shape
    np.testing.assert_array_equal(dev, dev2)
    same = float(np.mean(dev == host))
    assert same >= 0.999, f"only {same:.4%} of the quantiles equal the host ends' bit for bit"
    bar, _ = pb.bar(precision, lambda: model.forward(inp)[0], lambda o: per_quantile_err(o, exp), pb.TINY)
    err = per_quantile_err(dev, exp)
    assert err < bar, f"{precision}: per-quantile rel max err {err:.3e} (bar {bar:.3e})"


@pytest.mark.parametrize("case", ["covariates", "degenerate"])
def test_device_prep_tokens_match_the_oracle(jc, tiny, case):
    # jc_chronos2_prep_device (the norm and token kernels of jc_forecast_chronos2) against the C restatement of
    # ModelPrep.of (the reference's loop order, double sums): equal bit for bit but where a double log (CUDA's
    # against glibc's) lands within an ulp of a float rounding boundary
    torch = pytest.importorskip("torch")
    import ctypes

    from jitcast_b200 import _lib

    c, _, model = tiny
    inp = ends_input(c, case)
    ref = np.asarray(model.prepare(inp)["tokens"], np.float32)
    lay = c2.ModelLayout.of(c, inp)
    dev = torch.device("cuda", 0)
    win = torch.from_numpy(np.ascontiguousarray(lay.window, np.float32)).to(dev)
    fut = torch.from_numpy(np.ascontiguousarray(lay.future, np.float32)).to(dev)
    tok = torch.empty(ref.size, device=dev)
    stream = torch.cuda.current_stream(dev)
    _lib.check(_lib.lib().jc_chronos2_prep_device(0, lay.rows, lay.context_patches, lay.output_patches, c.patch_size,
                                                  win.data_ptr(), fut.data_ptr(),
                                                  float(np.float32(c.time_encoding_scale)), int(c.use_arcsinh),
                                                  tok.data_ptr(), ctypes.c_void_p(stream.cuda_stream)))
    torch.cuda.synchronize()
    got = tok.cpu().numpy().reshape(ref.shape)
    same = float(np.mean(got == ref))
    assert same >= 0.9999, f"only {same:.4%} of the tokens equal the oracle's bit for bit"
    np.testing.assert_allclose(got, ref, rtol=2.0 ** -22, atol=0)


@pytest.mark.parametrize("case", ["covariates", "degenerate"])
def test_device_finish_matches_the_oracle(jc, tiny, case):
    # jc_chronos2_finish_device on the oracle's raw output patch embedding against its ModelPrep.finish
    torch = pytest.importorskip("torch")
    import ctypes

    from jitcast_b200 import _lib

    c, _, model = tiny
    inp = ends_input(c, case)
    out, raw = model.forward(inp)
    prep = model.prepare(inp)
    ls = np.stack([prep["loc"], prep["scale"]], axis=1).astype(np.float32)
    dev = torch.device("cuda", 0)
    r = torch.from_numpy(np.ascontiguousarray(raw, np.float32)).to(dev)
    lsd = torch.from_numpy(np.ascontiguousarray(ls)).to(dev)
    got_t = torch.empty(out.size, device=dev)
    stream = torch.cuda.current_stream(dev)
    _lib.check(_lib.lib().jc_chronos2_finish_device(0, out.shape[0], inp.output_patches, c.patch_size,
                                                    c.num_quantiles, int(c.use_arcsinh), lsd.data_ptr(), r.data_ptr(),
                                                    got_t.data_ptr(), ctypes.c_void_p(stream.cuda_stream)))
    torch.cuda.synchronize()
    got = got_t.cpu().numpy().reshape(out.shape)
    same = float(np.mean(got == out))
    assert same >= 0.9999, f"only {same:.4%} of the quantiles equal the oracle's bit for bit"
    np.testing.assert_allclose(got, out, rtol=1e-6, atol=1e-6 * float(np.abs(out).max()))


def test_host_ends_device_entry_point_matches_host(jc, tiny):
    # jc_forecast_chronos2_device: window, future covariates and layout in HBM, quantiles written there
    torch = pytest.importorskip("torch")
    import ctypes

    from jitcast_b200 import _lib

    c, w, _ = tiny
    inp = mixed_input(c, covariate_groups=2)
    lay = c2.ModelLayout.of(c, inp)
    gs, ge = c2.group_ranges(lay.group)
    with c2.Chronos2Engine(c, w, precision="fp16") as eng:
        host = eng.forecast(lay, gs, ge)
        dev = torch.device("cuda", 0)
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dt)).to(dev)  # noqa: E731
        keep = dict(win=t(lay.window, np.float32), fut=t(lay.future, np.float32), live=t(lay.live, np.int32),
                    gs=t(gs, np.int32), ge=t(ge, np.int32))
        blk = c2.Block(lay.rows, lay.context_patches, lay.output_patches, None, keep["live"].data_ptr(),
                       keep["gs"].data_ptr(), keep["ge"].data_ptr())
        win = c2.Window(blk, keep["win"].data_ptr(), keep["fut"].data_ptr(), float(c.time_encoding_scale),
                        int(c.use_arcsinh))
        out = torch.empty(host.shape, device=dev)
        stream = torch.cuda.current_stream(dev)
        _lib.check(_lib.lib().jc_forecast_chronos2_device(eng.handle, 0, ctypes.byref(win), out.data_ptr(),
                                                          ctypes.c_void_p(stream.cuda_stream)))
        eng.sync()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), host)


def test_without_reg_token(jc):
    c = tiny_config(use_reg_token=False)
    w = c2.random_checkpoint(c, seed=6)
    inp = mixed_input(c, covariate_groups=1, length=200)
    exp, _ = oc2.Model(c, w).forward(inp)
    with c2.Chronos2Engine(c, w, precision="fp32") as eng:
        got = c2.B200Chronos2Forward(eng).forward(inp)
    assert per_quantile_err(got, exp) < pb.TINY["fp32"]


def test_bucketed_plans_match_exact_plans(jc, tiny):
    # plans are built for bucketed row counts (33-64 rows in steps of 8): inputs of 49 and 51 rows both run on a
    # 56-row plan whose padding rows are dummy series; every real row's outputs equal an exact-shape plan's
    c, w, _ = tiny
    with c2.Chronos2Engine(c, w, precision="bf16") as bucketed, c2.Chronos2Engine(c, w, precision="bf16") as exact:
        exact.set_option("buckets", 0)
        for series, seed, rows in ((42, 41, 49), (44, 42, 51)):
            inp = mixed_input(c, series=series, covariate_groups=5, seed=seed)
            assert len(inp.group) == rows
            got = c2.B200Chronos2Forward(bucketed).forward(inp)
            ref = c2.B200Chronos2Forward(exact).forward(inp)
            np.testing.assert_array_equal(got, ref)


def test_sharded_two_slots(jc, tiny):
    c, w, _ = tiny
    inp = mixed_input(c, series=9, covariate_groups=3)
    with c2.Chronos2Engine(c, w, devices=(0,), precision="fp32") as one, \
            c2.Chronos2Engine(c, w, devices=(0, 0), precision="fp32") as two:
        a = c2.B200Chronos2Forward(one).forward(inp)
        b = c2.B200Chronos2Forward(two).forward(inp)
    np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-6)


@pytest.fixture(scope="module")
def config2_case():
    """BASELINE config 2 (d 768, 12 layers, 128 context patches + [REG] + 4 future, 21 quantiles) on a few
    random-walk series, with the oracle's outputs."""
    c = c2.config2()
    w = c2.random_checkpoint(c, seed=0)
    series = 2
    x = workloads.random_walk(series, 2048, seed=0)
    inp = c2.ModelInput(x, np.arange(series, dtype=np.int32), 4)
    exp, _ = oc2.Model(c, w).forward(inp)
    return c, w, inp, exp


@pytest.mark.parametrize("precision", ["fp32", "tf32", "bf16", "fp16"])
def test_config2_full_size_matches_oracle(jc, config2_case, precision):
    c, w, inp, exp = config2_case
    bar, floor = pb.bar(precision, lambda: oc2.Model(c, w).forward(inp)[0], lambda o: per_quantile_err(o, exp))
    with c2.Chronos2Engine(c, w, precision=precision) as eng:
        got = c2.B200Chronos2Forward(eng).forward(inp)
    err = per_quantile_err(got, exp)
    print(f"config2 {precision}: per-quantile rel max err {err:.3e} (bar {bar:.3e}, reduced-precision oracle {floor})")
    assert err < bar, f"{precision}: per-quantile rel max err {err:.3e} (bar {bar:.3e})"
