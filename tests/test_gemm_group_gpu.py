"""Grouped GEMM launches (jc_gemm_group_device) against one jc_gemm_device call per problem.

A group runs the tiles of up to four independent GEMMs in one persistent launch. The cases are the ones the
forwards use: TiRex-2's headwise sLSTM gates (four K = 128 GEMMs over column windows of one input, into
column windows of one output: tirex2/tornado/TornadoForward.java:730) and a patch embedding's two GEMMs of one
input with different widths and epilogues (timestral/tornado/TimestralForward.java:327), plus ragged problems
small enough for the single-CTA kernel. Each problem's output must equal its own launch's bit for bit, in every
precision mode.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PRECISIONS = ["fp32", "tf32", "bf16", "fp16"]


def storage(x, precision):
    """(hi, lo): the fp32 CUDA tensor x in the precision's operand storage format."""
    import torch

    if precision == "bf16":
        return x.bfloat16(), None
    if precision == "fp16":
        return x.half(), None
    u = x.contiguous().view(torch.int32)
    hi = ((u + 0xFFF + ((u >> 13) & 1)) & ~0x1FFF).view(torch.float32)  # round to nearest TF32
    return hi, (x - hi if precision == "fp32" else None)


def build(case, precision, rng, dev):
    """(problems as (a_hi, a_lo, w_hi, w_lo, bias, flags, output index, first column), output shapes)."""
    import torch

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    probs = []
    if case == "gates":  # x [M, 4·128]: head h reads columns 128h.., writes columns 512h.. of one C [M, 2048]
        m = 8192
        x_hi, x_lo = storage(t(rng.standard_normal((m, 512))), precision)
        for h in range(4):
            w_hi, w_lo = storage(t(rng.standard_normal((512, 128)) / np.sqrt(128)), precision)
            win = slice(128 * h, 128 * h + 128)
            probs.append((x_hi[:, win], None if x_lo is None else x_lo[:, win], w_hi, w_lo, None, 0, 0, 512 * h))
        return probs, [(m, 2048)]
    if case == "embed":  # one input, hidden (bias, SiLU) and residual (bias) of different widths
        m = 20000
        a_hi, a_lo = storage(t(rng.standard_normal((m, 64))), precision)
        for i, (n, flags) in enumerate(((4096, 1 | 4), (1024, 1))):
            w_hi, w_lo = storage(t(rng.standard_normal((n, 64)) / 8), precision)
            probs.append((a_hi, a_lo, w_hi, w_lo, t(rng.uniform(-0.1, 0.1, n)), flags, i, 0))
        return probs, [(m, 4096), (m, 1024)]
    shapes = []  # ragged and small: the single-CTA kernel; += C and ReLU on two of them
    for i, (m, n, k, flags) in enumerate(((333, 200, 192, 0), (1000, 136, 64, 2), (77, 300, 256, 16))):
        a_hi, a_lo = storage(t(rng.standard_normal((m, k))), precision)
        w_hi, w_lo = storage(t(rng.standard_normal((n, k)) / np.sqrt(k)), precision)
        probs.append((a_hi, a_lo, w_hi, w_lo, None, flags, i, 0))
        shapes.append((m, n))
    return probs, shapes


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("case", ["gates", "embed", "ragged"])
def test_group_equals_separate_launches(jc, precision, case):
    import torch

    from jitcast_b200 import ops

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(len(case) * 7 + PRECISIONS.index(precision))
    probs, shapes = build(case, precision, rng, dev)
    c0 = [torch.from_numpy(rng.standard_normal(s).astype(np.float32)).to(dev) for s in shapes]
    c_sep = [c.clone() for c in c0]
    c_grp = [c.clone() for c in c0]
    sep, grp = [], []
    for a_hi, a_lo, w_hi, w_lo, bias, flags, oi, col0 in probs:
        n = w_hi.shape[0]
        sep.append(ops.problem(a_hi, w_hi, c_sep[oi][:, col0:col0 + n], flags, bias, a_lo, w_lo))
        grp.append(ops.problem(a_hi, w_hi, c_grp[oi][:, col0:col0 + n], flags, bias, a_lo, w_lo))
    stream = torch.cuda.current_stream(dev)
    for p in sep:
        ops.gemm_device(p, precision, stream=stream)
    ops.gemm_group_device(grp, precision, stream=stream)
    ops.device_sync(0)
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(c_sep, c_grp)):
        assert torch.isfinite(b).all()
        assert not torch.equal(b, c0[i]), f"{case} {precision}: output {i} untouched"
        assert torch.equal(a, b), f"{case} {precision}: output {i} of the grouped launch differs from separate launches"
