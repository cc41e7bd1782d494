"""jc_linear_device_noalloc, the allocation-free GEMM entry point, against jc_linear_device.

Callers that cannot allocate GPU memory while running (a fixed arena or budget, or code that must not
let cudaMalloc/cudaFree synchronise the device) use jc_linear_device_noalloc: it keeps its converted
operands in a fixed scratch array inside the library. This file checks, through the C ABI, that two
calls in a row give the same C as the allocating entry point, and that shapes too large for the fixed
scratch are refused. It is collected last so a failure here comes after every other test has run.
"""

import ctypes

import numpy as np
import pytest

from jitcast_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {_lib.FP32: 1e-4, _lib.TF32: 1e-3, _lib.BF16: 1e-2, _lib.FP16: 2e-3}


def _run(fn, prec, a, w, b, c, flags, stream):
    m, k = a.shape
    n = w.shape[0]
    st = fn(0, prec, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), b.data_ptr(), c.data_ptr(),
            c.stride(0), m, n, k, flags, stream)
    assert st == _lib.OK, _lib.last_error()


@pytest.mark.parametrize("prec", [_lib.BF16, _lib.TF32, _lib.FP32, _lib.FP16])
def test_noalloc_matches_allocating_entry_point(prec):
    import torch

    L = _lib.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.Stream(dev)
    rng = np.random.default_rng(prec)
    flags = _lib.BIAS | _lib.ACCUMULATE | _lib.SILU
    for m, n, k in [(1024, 768, 256), (333, 200, 70)]:  # two calls in a row, different shapes
        a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev)
        w = torch.from_numpy((rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)).to(dev)
        b = torch.from_numpy(rng.uniform(-0.1, 0.1, n).astype(np.float32)).to(dev)
        c0 = torch.from_numpy(rng.standard_normal((m, n)).astype(np.float32)).to(dev)
        c_ref, c_new = c0.clone(), c0.clone()
        torch.cuda.synchronize()
        _run(L.jc_linear_device, prec, a, w, b, c_ref, flags, stream.cuda_stream)
        assert L.jc_device_sync(0) == _lib.OK, _lib.last_error()
        _run(L.jc_linear_device_noalloc, prec, a, w, b, c_new, flags, stream.cuda_stream)
        torch.cuda.synchronize()
        ref = c_ref.cpu().numpy().astype(np.float64)
        got = c_new.cpu().numpy().astype(np.float64)
        err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6)
        assert err < TOL[prec], f"precision {prec} {m}x{n}x{k}: {err:.3e}"


def test_noalloc_refuses_shapes_beyond_its_scratch():
    L = _lib.lib()
    big = 1 << 14  # (16384 + 16384) x 16384 BF16 operands need far more than the fixed scratch
    dummy = ctypes.c_float()
    p = ctypes.addressof(dummy)
    st = L.jc_linear_device_noalloc(0, _lib.BF16, p, big, p, big, None, p, big, big, big, big, 0, None)
    assert st == _lib.ERR_UNSUPPORTED_SHAPE
    assert "fixed scratch" in _lib.last_error()
