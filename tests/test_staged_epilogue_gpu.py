"""The staged GEMM epilogues against the per-thread ones, bit for bit.

On CTA-pair tiles the residual GEMMs (wo, w3: C += A·Wᵀ in place), the q|k|v|gate GEMM (bias, RoPE, sigmoid
gate, 16-bit outputs), the SwiGLU GEMM and plain GEMMs with a 16-bit output (an FFN's hidden layer) move their
outputs through shared memory and out by TMA stores; ``JC_GEMM_STAGED=0`` keeps them on the epilogues that store
from registers. Both compute every value with the same arithmetic, so a forward must come out identical either
way: Timestral (d 256, 4 heads of 64, 2 layers, 2,000 series: M = 260,000 rows per GEMM) and Chronos-2 config 2
(400 series: M = 53,600 rows; its ReLU FFN is a plain 16-bit-output GEMM). The switch is read once per process, so
each side runs in a child process.
"""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from jitcast_b200 import timestral as ts
from jitcast_b200 import workloads
prec, out = sys.argv[2], sys.argv[3]
c = ts.TimestralConfig(patch_size=32, d_model=256, num_heads=4, mlp_hidden_dim=1024, block_schedule=["time"] * 2,
                       quantile_knots=ts.default_knots(21), block_size=16, context_length=4096).validate()
w = ts.random_checkpoint(c, seed=1)
x = workloads.sinusoid_noise(2000, 4096, seed=3)
block = ts.BlockInput(x, np.ones_like(x, bool), np.arange(2000, dtype=np.int32), 2)
dev = torch.device("cuda", 0)
stream = torch.cuda.Stream(dev)
with ts.TimestralEngine(c, w, precision=prec) as eng:
    dw = ts.DeviceWindow(ts.WindowInputs.of(c, ts.BlockLayout.of(c, block)), dev)
    o = torch.empty(dw.out_shape(c), device=dev)
    dw.forecast(eng, o, stream)
    eng.sync()
    torch.cuda.synchronize()
    np.save(out, o.cpu().numpy())
"""


CHILD_C2 = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from jitcast_b200 import chronos2 as c2
from jitcast_b200 import workloads
prec, out = sys.argv[2], sys.argv[3]
c = c2.config2()
w = c2.random_checkpoint(c, seed=0)
x = workloads.random_walk(400, 2048, seed=1)
inp = c2.ModelInput(x, np.arange(400, dtype=np.int32), 4)
with c2.Chronos2Engine(c, w, precision=prec) as eng:
    np.save(out, np.asarray(c2.B200Chronos2Forward(eng).forward(inp)))
"""


def forecast(tmp_path, child, prec, staged):
    out = tmp_path / f"{prec}_{staged}.npy"
    env = dict(os.environ, JC_GEMM_STAGED="1" if staged else "0")
    r = subprocess.run([sys.executable, "-c", child, str(ROOT), prec, str(out)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.load(out)


@pytest.mark.parametrize("model", ["timestral", "chronos2"])
@pytest.mark.parametrize("prec", ["fp16", "bf16"])
def test_staged_epilogues_equal_register_epilogues(jc, tmp_path, model, prec):
    child = CHILD if model == "timestral" else CHILD_C2
    staged = forecast(tmp_path, child, prec, True)
    plain = forecast(tmp_path, child, prec, False)
    assert np.isfinite(staged).all()
    assert np.array_equal(staged, plain), f"{model} {prec}: max |diff| {np.abs(staged - plain).max():.3e}"
