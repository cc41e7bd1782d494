"""jc_linear_device_noalloc, the allocation-free GEMM entry point, against jc_linear_device and the oracle.

Callers that cannot allocate GPU memory while running (a fixed arena or budget, or code that must not
let cudaMalloc/cudaFree synchronise the device) use jc_linear_device_noalloc: it keeps its converted
operands in a fixed scratch array inside the library. This file checks, through the C ABI, that two
calls in a row give the same C as the allocating entry point and as the C restatement of the reference's
Kernels.gemm semantics (oracle.gemm), on the single-CTA and the CTA-pair kernels; that a call after the
first allocates no device memory; and that shapes too large for the fixed scratch are refused. It is
collected last so a failure here comes after every other test has run.
"""

import ctypes

import numpy as np
import pytest

import oracle
from jitcast_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {_lib.FP32: 1e-4, _lib.TF32: 1e-3, _lib.BF16: 1e-2, _lib.FP16: 2e-3}
# (m, n, k): the single-CTA kernel, a ragged shape, and 2560 x 2048 (80 tiles of 256 x 256: the CTA-pair
# kernel) whose 16-bit and TF32 operands still fit the fixed scratch (JC_FP32's hi/lo pairs do not)
SHAPES = [(1024, 768, 256), (333, 200, 70), (2560, 2048, 512)]


def _run(fn, prec, a, w, b, c, flags, stream):
    m, k = a.shape
    n = w.shape[0]
    st = fn(0, prec, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), b.data_ptr(), c.data_ptr(),
            c.stride(0), m, n, k, flags, stream)
    assert st == _lib.OK, _lib.last_error()


def _rel(got, ref):
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6)


@pytest.mark.parametrize("prec", [_lib.BF16, _lib.TF32, _lib.FP32, _lib.FP16])
def test_noalloc_matches_allocating_entry_point(prec):
    import torch

    L = _lib.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.Stream(dev)
    rng = np.random.default_rng(prec)
    flags = _lib.BIAS | _lib.ACCUMULATE | _lib.SILU
    shapes = SHAPES[:2] if prec == _lib.FP32 else SHAPES
    for m, n, k in shapes:  # calls in a row, different shapes
        a_h = rng.standard_normal((m, k)).astype(np.float32)
        w_h = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
        b_h = rng.uniform(-0.1, 0.1, n).astype(np.float32)
        c0_h = rng.standard_normal((m, n)).astype(np.float32)
        a, w, b, c0 = (torch.from_numpy(v).to(dev) for v in (a_h, w_h, b_h, c0_h))
        c_ref, c_new = c0.clone(), c0.clone()
        torch.cuda.synchronize()
        _run(L.jc_linear_device, prec, a, w, b, c_ref, flags, stream.cuda_stream)
        assert L.jc_device_sync(0) == _lib.OK, _lib.last_error()
        _run(L.jc_linear_device_noalloc, prec, a, w, b, c_new, flags, stream.cuda_stream)
        torch.cuda.synchronize()
        ref = c_ref.cpu().numpy().astype(np.float64)
        got = c_new.cpu().numpy().astype(np.float64)
        err = _rel(got, ref)
        assert err < TOL[prec], f"precision {prec} {m}x{n}x{k}: {err:.3e} against jc_linear_device"
        exp = oracle.gemm(a_h, w_h, b_h, c0_h, flags).astype(np.float64)
        err_o = _rel(got, exp)
        assert err_o < TOL[prec], f"precision {prec} {m}x{n}x{k}: {err_o:.3e} against the oracle"


def test_noalloc_call_allocates_no_device_memory():
    import torch

    L = _lib.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.Stream(dev)
    rng = np.random.default_rng(3)
    m, n, k = 2560, 2048, 512
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev)
    w = torch.from_numpy((rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)).to(dev)
    b = torch.from_numpy(rng.uniform(-0.1, 0.1, n).astype(np.float32)).to(dev)
    c = torch.zeros((m, n), device=dev)
    # the first call on the device loads the module (and with it the fixed scratch); later calls on new
    # shapes and precisions must leave the device's free memory where it was
    _run(L.jc_linear_device_noalloc, _lib.BF16, a[:64, :64], w[:64, :64], b, c, _lib.BIAS, stream.cuda_stream)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(dev)
    for prec in (_lib.BF16, _lib.FP16, _lib.TF32):
        _run(L.jc_linear_device_noalloc, prec, a, w, b, c, _lib.BIAS | _lib.RELU, stream.cuda_stream)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(dev)
    assert free_after == free_before, f"free device memory moved by {free_before - free_after} bytes"


def test_noalloc_refuses_shapes_beyond_its_scratch():
    L = _lib.lib()
    dummy = ctypes.c_float()
    p = ctypes.addressof(dummy)
    big = 1 << 14  # (16384 + 16384) x 16384 BF16 operands need far more than the fixed scratch
    st = L.jc_linear_device_noalloc(0, _lib.BF16, p, big, p, big, None, p, big, big, big, big, 0, None)
    assert st == _lib.ERR_UNSUPPORTED_SHAPE
    assert "fixed scratch" in _lib.last_error()
    # m and k near INT_MAX: the size check must refuse them rather than wrap its byte count
    huge = 2**31 - 1
    st = L.jc_linear_device_noalloc(0, _lib.FP32, p, huge, p, huge, None, p, 1, huge, 1, huge, 0, None)
    assert st == _lib.ERR_UNSUPPORTED_SHAPE
    assert "fixed scratch" in _lib.last_error()
