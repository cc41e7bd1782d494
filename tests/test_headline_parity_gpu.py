"""Parity at the shape the headline benchmark runs.

bench.py times the config-3 model (d 1024, 16 layers, 128 context + 2 decoder tokens, 21 quantiles) over
8,192-series chunks of the seeded sinusoid + noise workload through ``jc_forecast_timestral_device``: M =
1,064,960 rows per GEMM, on the CTA-pair (256 × 256 tile) kernel. Here one such chunk (chunk seed 0, the
bench's first) runs through that same entry point, and sampled series — the first, the last and two interior
ones — are compared with the C restatement of the reference's FP32 CPU forward (CpuTimestral.predictBlock,
CpuTimestral.java:87-314) run on those series alone. Series are independent (each is a group of its own), so
the oracle's forecast of a series does not depend on the batch around it.

This follows the reference's batch-parity check (TimestralBatchParityAccelTest.java:49-130: the CPU forward and
the device forward on the same inputs at batch size), with the error measure max|a − e| / max|e| taken on every
quantile level (TimestralGolden.java:125-140).
"""

import os

import numpy as np
import pytest

from jitcast_b200 import timestral as ts
from jitcast_b200 import workloads
from oracle import timestral as ots

pytestmark = pytest.mark.gpu

CHUNK = 8192
SAMPLE = (0, 2730, 5461, CHUNK - 1)
# the FP32-accumulate mode 1e-3, the 16-bit tensor-core mode 1e-2
BAR = {"fp32": 1e-3, "fp16": 1e-2}


def per_quantile_err(actual, expected):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert np.isfinite(a).all()
    return max(np.abs(a[..., k] - e[..., k]).max() / max(np.abs(e[..., k]).max(), 1e-6)
               for k in range(e.shape[-1]))


@pytest.fixture(scope="module")
def headline():
    c = ts.config3()
    w = ts.random_checkpoint(c, seed=0)
    x = workloads.sinusoid_noise(CHUNK, 4096, seed=0)  # bench.py's first chunk
    block = ts.BlockInput(x, np.ones_like(x, bool), np.arange(CHUNK, dtype=np.int32), 2)
    xs = x[list(SAMPLE)]
    sample = ts.BlockInput(xs, np.ones_like(xs, bool), np.arange(len(SAMPLE), dtype=np.int32), 2)
    exp, _ = ots.Model(c, w).predict_block(sample, nthreads=os.cpu_count())
    return c, w, block, exp


@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_headline_chunk_matches_oracle(jc, headline, precision):
    import torch

    c, w, block, exp = headline
    dev = torch.device("cuda", 0)
    lay = ts.BlockLayout.of(c, block)
    assert lay.rows == CHUNK and lay.tokens == 130
    stream = torch.cuda.Stream(dev)
    with ts.TimestralEngine(c, w, precision=precision) as eng:
        dw = ts.DeviceWindow(ts.WindowInputs.of(c, lay), dev)
        out = torch.empty(dw.out_shape(c), device=dev)
        dw.forecast(eng, out, stream)
        eng.sync()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
    assert np.isfinite(got).all()
    err = per_quantile_err(got[list(SAMPLE)], exp)
    print(f"headline chunk {precision}: per-quantile rel max err {err:.3e} over series {SAMPLE}")
    assert err < BAR[precision], f"{precision}: per-quantile rel max err {err:.3e}"
