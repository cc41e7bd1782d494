"""The time-attention kernels through the C ABI (jc_time_attention_device) against a plain PyTorch FP32
masked-softmax attention of the same op, on random q/k/v, gates and masks.

Covers the token counts the models produce and the tcgen05 kernel's edges: fewer tokens than the
128-query MMA tile (rows of the tile past n belong to the next row), exactly 128, the Timestral 130 (two
decoder queries past the tile), the Chronos-2 133 (five), and up to the 256-token limit; both mask modes
(BlockLayout.timeAllowed with known covariates and key gaps; Chronos-2 liveness with dead keys and a fully
dead row). Bars (max |a − e| / max |e|): the FP32-math CUDA-core kernel 1e-5 on FP32 buffers; the 16-bit
kernels 4e-3 (FP16, 11-bit probabilities) and 2e-2 (BF16, 8-bit probabilities), from their own operand
rounding.
"""

import ctypes

import numpy as np
import pytest

from jitcast_b200 import _lib

pytestmark = pytest.mark.gpu

PREC = {"fp32": (_lib.FP32, "float32"), "bf16": (_lib.BF16, "bfloat16"), "fp16": (_lib.FP16, "float16")}
TOL = {"fp32": 1e-5, "bf16": 2e-2, "fp16": 4e-3}


def make_case(torch, rows, n, heads, mode, seed, gated=True, enc=None):
    g = torch.Generator().manual_seed(seed)
    d = heads * 64
    qkv = torch.randn(rows * n, 3 * d, generator=g)
    gate = torch.rand(rows * n, d, generator=g) if gated else None
    if mode == 0:
        enc = enc if enc is not None else max(1, n - 2)
        ll = max(0, enc - 3)
        key_valid = (torch.rand(rows, enc, generator=g) > 0.2).int()
        known = (torch.rand(rows, generator=g) > 0.6).int()
        return dict(qkv=qkv, gate=gate, enc=enc, ll=ll, key_valid=key_valid, known=known, live=None)
    live = (torch.rand(rows, n, generator=g) > 0.25).int()
    live[0] = 0  # a row with no live key attends nothing: zeros
    return dict(qkv=qkv, gate=gate, enc=n, ll=n, key_valid=None, known=None, live=live)


def allowed_mask(torch, c, rows, n, mode):
    q = torch.arange(n)[:, None]
    k = torch.arange(n)[None, :]
    if mode == 1:
        return c["live"].bool()[:, None, :].expand(rows, n, n)
    enc, ll = c["enc"], c["ll"]
    valid = torch.zeros(rows, n, dtype=torch.bool)
    valid[:, :enc] = c["key_valid"].bool()
    known = c["known"].bool()[:, None, None]
    v = valid[:, None, :]
    enc_q = (k < enc) & ((k == q) | (v & ((k <= q) | known)))
    dec_q = torch.where(k < enc, (k < ll) & v, (k <= q) & (k < n))
    return torch.where(q < enc, enc_q, dec_q)


def reference(torch, c, rows, n, heads, scale, mode, dtype):
    d = heads * 64
    x = c["qkv"].to(dtype).float().view(rows, n, 3, heads, 64)
    q, k, v = x[:, :, 0], x[:, :, 1], x[:, :, 2]
    s = torch.einsum("rqhe,rkhe->rhqk", q, k) * scale
    m = allowed_mask(torch, c, rows, n, mode)[:, None]
    s = s.masked_fill(~m, float("-inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    o = torch.einsum("rhqk,rkhe->rqhe", p, v).reshape(rows * n, d)
    if c["gate"] is not None:
        o = o * c["gate"].to(dtype).float()
    return o


def run(torch, c, rows, n, heads, scale, mode, prec, cuda_cores=False):
    code, tname = PREC[prec]
    dt = getattr(torch, tname)
    dev = torch.device("cuda", 0)
    d = heads * 64
    qkv = c["qkv"].to(dt).to(dev).contiguous()
    gate = None if c["gate"] is None else c["gate"].to(dt).to(dev).contiguous()
    out = torch.full((rows * n, d), float("nan"), dtype=dt, device=dev)
    kv = None if c["key_valid"] is None else c["key_valid"].int().to(dev).contiguous()
    kn = None if c["known"] is None else c["known"].int().to(dev).contiguous()
    lv = None if c["live"] is None else c["live"].int().to(dev).contiguous()
    ptr = lambda t: None if t is None else t.data_ptr()
    _lib.check(_lib.lib().jc_time_attention_device(
        0, code, qkv.data_ptr(), 3 * d, ptr(gate), d, out.data_ptr(), d, rows, n, heads, 64, d, scale, mode,
        c["enc"], c["ll"], ptr(kv), ptr(kn), ptr(lv), _lib.ATTN_CUDA_CORES if cuda_cores else 0,
        ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
    _lib.check(_lib.lib().jc_device_sync(0))
    return out.float().cpu()


def rel_err(a, e):
    assert not torch_isnan(a)
    return float((a - e).abs().max() / max(float(e.abs().max()), 1e-6))


def torch_isnan(t):
    return bool(t.isnan().any())


@pytest.mark.parametrize("n", [18, 128, 130, 133, 200, 256])
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("prec", ["fp16", "bf16"])
def test_tensor_core_attention_matches_torch(jc, n, mode, prec):
    torch = pytest.importorskip("torch")
    rows, heads = 3, 2
    scale = 0.125 if mode == 0 else 1.0
    c = make_case(torch, rows, n, heads, mode, seed=n * 10 + mode)
    exp = reference(torch, c, rows, n, heads, scale, mode, getattr(torch, PREC[prec][1]))
    got = run(torch, c, rows, n, heads, scale, mode, prec)
    err = rel_err(got, exp)
    print(f"n={n} mode={mode} {prec}: rel max err {err:.2e}")
    assert err < TOL[prec], f"n={n} mode={mode} {prec}: rel max err {err:.3e}"


@pytest.mark.parametrize("n,mode", [(130, 0), (133, 1)])
def test_cuda_core_attention_fp32_matches_torch(jc, n, mode):
    torch = pytest.importorskip("torch")
    rows, heads = 2, 2
    scale = 0.125
    c = make_case(torch, rows, n, heads, mode, seed=7)
    exp = reference(torch, c, rows, n, heads, scale, mode, torch.float32)
    got = run(torch, c, rows, n, heads, scale, mode, "fp32", cuda_cores=True)
    assert rel_err(got, exp) < TOL["fp32"]


def test_encoder_longer_than_the_tile(jc):
    # enc = 200 > 128: encoder queries past the MMA tile run on the CUDA cores with the encoder mask
    torch = pytest.importorskip("torch")
    rows, heads, n = 2, 2, 210
    c = make_case(torch, rows, n, heads, 0, seed=3, enc=200)
    exp = reference(torch, c, rows, n, heads, 0.125, 0, torch.float16)
    got = run(torch, c, rows, n, heads, 0.125, 0, "fp16")
    assert rel_err(got, exp) < TOL["fp16"]


@pytest.mark.parametrize("n,enc", [(64, 60), (129, 128), (130, 128), (136, 128), (131, 125)])
@pytest.mark.parametrize("prec", ["fp16", "bf16"])
def test_timestral_layout_many_rows(jc, n, enc, prec):
    # the Timestral layout (mask mode 0) over many rows and heads, known rows and key gaps included: 1 to 8 decoder
    # queries past the MMA tile, an encoder that is not a multiple of 16, a row shorter than the tile
    torch = pytest.importorskip("torch")
    rows, heads = 150, 8
    c = make_case(torch, rows, n, heads, 0, seed=n + enc, enc=enc)
    exp = reference(torch, c, rows, n, heads, 0.125, 0, getattr(torch, PREC[prec][1]))
    got = run(torch, c, rows, n, heads, 0.125, 0, prec)
    err = rel_err(got, exp)
    print(f"timestral layout n={n} enc={enc} {prec}: rel max err {err:.2e}")
    assert err < TOL[prec], f"n={n} enc={enc} {prec}: rel max err {err:.3e}"
