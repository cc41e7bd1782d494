"""The tcgen05 GEMM through the C ABI against the oracle, on a B200.

Cases follow the reference's own GEMM tests (tornado/KernelsAccelTest.java:57-149: Random(7)
inputs, ragged 37×45×70, 150×200×88 and 150×300×88 with element offsets, every flag set) with its
error measure (relative max error, KernelHarness.java:104-117), plus BASELINE config 1 and shapes
that exercise every tile width, multi-stage K loops and the persistent tile walk.

Tolerances: FP32 (3×TF32) 1e-4 — the reference's FP32 bar; TF32 1e-3 and BF16 1e-2 — the bars
BASELINE.json sets for the reduced-precision modes; FP16 2e-3 (11-bit mantissa).
"""

from pathlib import Path

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-4, "tf32": 1e-3, "bf16": 1e-2, "fp16": 2e-3}
GOLDEN = np.load(Path(__file__).parent / "golden" / "kernels_gemm.npz")
CASES = ["every_flag", "blocked", "blocked_wide"]


@pytest.mark.parametrize("precision", ["fp32", "tf32", "bf16", "fp16"])
@pytest.mark.parametrize("case", CASES)
def test_kernels_accel_cases(jc, case, precision):
    a, w, b, c0 = (GOLDEN[f"{case}/{k}"] for k in ("a", "w", "bias", "c0"))
    for f in GOLDEN[f"{case}/flags"]:
        f = int(f)
        got = jc.ops.gemm(a, w, b, c0, f, precision=precision)
        err = oracle.rel_max_err(got, GOLDEN[f"{case}/exp_{f}"])
        assert err < TOL[precision], f"{case} flags={f} {precision}: rel max err {err:.3e}"


def config1(seed=0):
    """M=1024 (16 series × 64 patch tokens), K=256, N=768; x~N(0,1),
    W~N(0,1/K), b~U(-0.1,0.1), seed 0."""
    rng = np.random.default_rng(seed)
    m, k, n = 1024, 256, 768
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    return x, w, b


@pytest.mark.parametrize("precision", ["fp32", "tf32", "bf16", "fp16"])
def test_config1_host(jc, precision):
    x, w, b = config1()
    got = jc.ops.linear(x, w, b, precision=precision)
    err = oracle.rel_max_err(got, oracle.linear(x, w, b))
    assert err < TOL[precision], f"{precision}: {err:.3e}"


@pytest.mark.parametrize("flags", [32 | 1, 4 | 16 | 1, 2])
def test_other_activations(jc, flags):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((70, 96), np.float32)
    w = (rng.standard_normal((130, 96)) * 0.2).astype(np.float32)
    b = rng.standard_normal(130).astype(np.float32)
    c0 = rng.standard_normal((70, 130)).astype(np.float32)
    got = jc.ops.gemm(a, w, b, c0, flags, precision="fp32")
    err = oracle.rel_max_err(got, oracle.gemm(a, w, b, c0, flags))
    assert err < 1e-4


@pytest.mark.parametrize("precision", ["fp32", "tf32", "bf16", "fp16"])
@pytest.mark.parametrize("m,n,k", [(1024, 768, 256),      # config 1
                                   (10240, 256, 128),     # 128-wide tiles
                                   (2053, 2304, 768),     # 256-wide tiles, M tail, persistent walk
                                   (1000, 1000, 1000)])   # ragged everything, 16 K stages
def test_device_buffers(jc, precision, m, n, k):
    import torch

    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    dev = torch.device("cuda:0")
    tx, tw, tb = (torch.from_numpy(v).to(dev) for v in (x, w, b))
    tc = torch.from_numpy(c0).to(dev)
    jc.ops.linear_device(tx, tw, tb, tc, jc.ops.BIAS | jc.ops.ACCUMULATE | jc.ops.SILU, precision=precision)
    jc.ops.device_sync(0)
    got = tc.cpu().numpy()
    exp = oracle.gemm(x, w, b, c0, jc.ops.BIAS | jc.ops.ACCUMULATE | jc.ops.SILU)
    err = oracle.rel_max_err(got, exp)
    assert err < TOL[precision], f"{precision} {m}x{n}x{k}: {err:.3e}"


@pytest.mark.parametrize("precision", ["tf32", "bf16", "fp16"])
@pytest.mark.parametrize("m,n,k,flags", [(4133, 4160, 1000, 0),          # CTA-pair tiles, ragged M, N and K
                                         (8192, 1024, 4096, 2),          # residual add, long K
                                         (9000, 1000, 1024, 2),          # residual add, ragged M and N
                                         (20000, 200, 512, 1 | 2),       # bias + residual, N below one tile
                                         (19000, 768, 256, 1 | 4)])      # bias + SiLU, short K
def test_cta_pair_tiles(jc, precision, m, n, k, flags):
    # shapes with at least one 256 × 256 tile per SM pair run on the two-CTA (cta_group::2) kernel; the residual
    # adds run its staged epilogue (TMA boxes of the residual, clipped at the ragged edges)
    import torch

    rng = np.random.default_rng(m + n + k + flags)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    dev = torch.device("cuda:0")
    tx, tw, tb, tc = (torch.from_numpy(v).to(dev) for v in (x, w, b, c0))
    jc.ops.linear_device(tx, tw, tb, tc, flags, precision=precision)
    jc.ops.device_sync(0)
    got = tc.cpu().numpy()
    exp = (torch.from_numpy(x).double() @ torch.from_numpy(w).double().T)
    if flags & 1:
        exp = exp + torch.from_numpy(b).double()
    if flags & 4:
        exp = exp * torch.sigmoid(exp)
    if flags & 2:
        exp = exp + torch.from_numpy(c0).double()
    err = oracle.rel_max_err(got, exp.numpy())
    assert err < TOL[precision], f"{precision} {m}x{n}x{k} flags {flags}: {err:.3e}"


def test_repeated_calls_reuse_scratch(jc):
    # growing and shrinking shapes through the same scratch slots, results stay exact
    for m, n, k in [(64, 64, 64), (700, 300, 520), (33, 17, 9), (700, 300, 520)]:
        rng = np.random.default_rng(m * n)
        a = rng.standard_normal((m, k)).astype(np.float32)
        w = rng.standard_normal((n, k)).astype(np.float32)
        got = jc.ops.gemm(a, w, None, None, 0, precision="fp32")
        assert oracle.rel_max_err(got, oracle.linear(a, w)) < 1e-4
