"""The oracle, pinned: java.util.Random known answers, and the C restatement of Ops.linear /
Kernels.gemm against the committed golden fixtures (bit-exact)."""

import numpy as np
import pytest

import oracle
from oracle import JavaRandom

GOLDEN = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "kernels_gemm.npz")
CASES = ["every_flag", "blocked", "blocked_wide"]


def test_java_random_known_answers():
    # Values of the Java platform's own Random for these seeds (its specified LCG and polar method).
    assert JavaRandom(42)._next(32) == -1170105035
    r = JavaRandom(42)
    assert r.next_gaussian() == pytest.approx(1.1419053154730547, abs=1e-15)
    assert JavaRandom(0).next_double() == pytest.approx(0.730967787376657, abs=1e-15)


def test_fixture_inputs_are_random7_draws():
    a = JavaRandom(7).gaussians(37 * 70, 1.0).reshape(37, 70)
    np.testing.assert_array_equal(a, GOLDEN["every_flag/a"])


@pytest.mark.parametrize("case", CASES)
def test_oracle_gemm_bit_exact(case):
    a, w, b, c0 = (GOLDEN[f"{case}/{k}"] for k in ("a", "w", "bias", "c0"))
    for f in GOLDEN[f"{case}/flags"]:
        got = oracle.gemm(a, w, b, c0, int(f), nthreads=4)
        np.testing.assert_array_equal(got, GOLDEN[f"{case}/exp_{int(f)}"], err_msg=f"{case} flags={f}")


def test_oracle_linear_thread_count_invariant():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((97, 33), np.float32)
    w = rng.standard_normal((29, 33), np.float32)
    b = rng.standard_normal(29, np.float32)
    y1 = oracle.linear(x, w, b, nthreads=1)
    y8 = oracle.linear(x, w, b, nthreads=8)
    np.testing.assert_array_equal(y1, y8)
    np.testing.assert_allclose(y1, x.astype(np.float64) @ w.T.astype(np.float64) + b, rtol=1e-5, atol=1e-5)


def test_oracle_rmsnorm():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 64), np.float32)
    g = rng.standard_normal(64, np.float32)
    y = oracle.rmsnorm(x, g, 1e-6)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * g
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)


def test_rel_max_err_definition():
    e = np.array([1.0, -4.0, 2.0])
    assert oracle.rel_max_err(e + [0, 0.4, 0], e) == pytest.approx(0.1)
    assert oracle.rel_max_err(np.array([np.nan, 0, 0]), e) == float("inf")


def test_sign_flip_complement():
    from jitcast_b200 import timestral as ts

    comp = ts.sign_flip_complement(ts.default_knots(9))
    assert list(comp) == list(range(8, -1, -1))
    with pytest.raises(ValueError):
        ts.sign_flip_complement([0.1, 0.5, 0.8])


def test_operand_rounding_matches_the_formats():
    # oracle.operand_format (a reduced-precision run of the reference arithmetic): BF16 and FP16 rounding equal
    # torch's conversions bit for bit over a wide range of magnitudes (FP16 saturating at ±65504, subnormals
    # kept); TF32 equals round-to-nearest-even at 10 mantissa bits
    import torch

    L = oracle.lib()
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(20000) * np.exp(rng.uniform(-22, 14, 20000))).astype(np.float32)
    v[:4] = [0.0, -0.0, 65519.0, -70000.0]
    for name, dt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        got = np.array([L.jco_round_operand(float(x), oracle.OPERAND_FORMATS[name]) for x in v], np.float32)
        src = np.clip(v, -65504, 65504) if name == "fp16" else v
        exp = torch.from_numpy(src).to(dt).float().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), exp.view(np.uint32))
    u = v.view(np.uint32).astype(np.uint64)
    exp = ((u + 0xFFF + ((u >> 13) & 1)) >> 13 << 13).astype(np.uint32).view(np.float32)
    got = np.array([L.jco_round_operand(float(x), oracle.OPERAND_FORMATS["tf32"]) for x in v], np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_operand_format_rounds_every_linear_and_is_restored():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((40, 96)).astype(np.float32)
    w = rng.standard_normal((24, 96)).astype(np.float32)
    exact = oracle.linear(x, w)
    with oracle.operand_format("bf16"):
        reduced = oracle.linear(x, w)
    import torch

    xb = torch.from_numpy(x).bfloat16().double().numpy()
    wb = torch.from_numpy(w).bfloat16().double().numpy()
    np.testing.assert_array_equal(reduced, (xb @ wb.T).astype(np.float32))
    np.testing.assert_array_equal(oracle.linear(x, w), exact)  # the reference's arithmetic again
    assert oracle.lib().jco_operand_format() == 0
