"""Op-level host API: the reference's shared GEMM operator on the B200 engine.

``gemm`` mirrors ``Kernels.gemm`` (tornado/Kernels.java:59-102): ``C[m, n] (+)= act(A·Wᵀ + b)``
with the same flag values and epilogue order (bias → SiLU/ReLU → += C), on host arrays.
``linear`` mirrors ``Ops.linear`` (cpu/Ops.java:33-51). ``linear_device`` runs on tensors that
already live in HBM (torch CUDA tensors), enqueued on the current torch stream.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import ACCUMULATE, BIAS, GELU, RELU, SILU, TWIN_ONLY, check, precision_code

__all__ = ["gemm", "linear", "linear_device", "gemm_device", "gemm_group_device", "GemmProblem", "device_sync", "BIAS",
           "ACCUMULATE", "SILU", "RELU", "GELU", "TWIN_ONLY"]


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def gemm(a, w, bias, c, flags: int, precision="bf16", device: int = 0) -> np.ndarray:
    """``C (+)= act(A·Wᵀ + b)`` with Kernels.gemm flags. ``a`` [m, k], ``w`` [n, k], ``bias`` [n] or
    None, ``c`` [m, n] (read with ACCUMULATE) or None. Returns the new C (a fresh array)."""
    a = _f32(a)
    w = _f32(w)
    if a.ndim != 2 or w.ndim != 2 or a.shape[1] != w.shape[1]:
        raise ValueError(f"shapes a{a.shape} w{w.shape} do not form A·Wᵀ")
    m, k = a.shape
    n = w.shape[0]
    out = np.zeros((m, n), np.float32) if c is None else np.array(c, np.float32, copy=True).reshape(m, n)
    b = None if bias is None else _f32(bias)
    if b is not None and b.shape != (n,):
        raise ValueError(f"bias shape {b.shape} != ({n},)")
    st = _lib.lib().jc_linear(device, precision_code(precision), a.ctypes.data, w.ctypes.data,
                              None if b is None else b.ctypes.data, out.ctypes.data, m, n, k, flags)
    check(st)
    return out


def linear(x, w, b=None, precision="bf16", device: int = 0) -> np.ndarray:
    """``Ops.linear``: y [rows, out] = x [rows, in] · w [out, in]ᵀ + b."""
    return gemm(x, w, b, None, BIAS if b is not None else 0, precision, device)


def linear_device(a, w, bias, c, flags: int, precision="bf16", stream=None) -> None:
    """The same GEMM on torch CUDA tensors (fp32; 2-D, unit stride in the last dimension), in place on
    ``c``, enqueued on ``stream`` (default: torch's current stream)."""
    import torch

    for name, t in (("a", a), ("w", w), ("c", c)):
        if t.dtype != torch.float32 or not t.is_cuda or t.dim() != 2 or t.stride(1) != 1:
            raise ValueError(f"{name} must be a 2-D fp32 CUDA tensor with unit column stride")
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or tuple(c.shape) != (m, n):
        raise ValueError("shapes do not form C[m, n] = A[m, k]·W[n, k]ᵀ")
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous() or bias.numel() != n):
        raise ValueError("bias must be a contiguous fp32 CUDA tensor of n elements")
    s = stream if stream is not None else torch.cuda.current_stream(a.device)
    st = _lib.lib().jc_linear_device(a.device.index, precision_code(precision), a.data_ptr(), a.stride(0),
                                     w.data_ptr(), w.stride(0), None if bias is None else bias.data_ptr(),
                                     c.data_ptr(), c.stride(0), m, n, k, flags, s.cuda_stream)
    check(st)


class GemmProblem(ctypes.Structure):
    """jc_gemm_problem: one GEMM of a group, on device operands in the precision's storage format."""

    _fields_ = [("a_hi", ctypes.c_void_p), ("a_lo", ctypes.c_void_p), ("lda", ctypes.c_longlong),
                ("w_hi", ctypes.c_void_p), ("w_lo", ctypes.c_void_p), ("ldw", ctypes.c_longlong),
                ("bias", ctypes.c_void_p), ("c", ctypes.c_void_p), ("ldc", ctypes.c_longlong), ("m", ctypes.c_int),
                ("n", ctypes.c_int), ("k", ctypes.c_int), ("flags", ctypes.c_int)]


def problem(a_hi, w_hi, c, flags: int = 0, bias=None, a_lo=None, w_lo=None) -> GemmProblem:
    """A GemmProblem over torch CUDA tensors: ``a_hi`` [m, k] and ``w_hi`` [n, k] (row views, unit column stride)
    in the storage format (bf16 / fp16 / fp32 holding TF32; JC_FP32 adds the fp32 remainders ``a_lo``, ``w_lo``),
    ``c`` [m, n] fp32, ``bias`` [n] fp32 or None."""
    m, k = a_hi.shape
    n = w_hi.shape[0]
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    return GemmProblem(ptr(a_hi), ptr(a_lo), a_hi.stride(0), ptr(w_hi), ptr(w_lo), w_hi.stride(0), ptr(bias),
                       c.data_ptr(), c.stride(0), m, n, k, flags)


def gemm_device(p: GemmProblem, precision="bf16", device: int = 0, stream=None) -> None:
    """``jc_gemm_device`` for one problem, enqueued on ``stream`` (default: torch's current stream)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream(device)
    check(_lib.lib().jc_gemm_device(device, precision_code(precision), p.a_hi, p.a_lo, p.lda, p.w_hi, p.w_lo, p.ldw,
                                    p.bias, p.c, p.ldc, p.m, p.n, p.k, p.flags, s.cuda_stream))


def gemm_group_device(problems, precision="bf16", device: int = 0, stream=None) -> None:
    """``jc_gemm_group_device``: 1 to 4 independent problems as one launch, enqueued on ``stream``."""
    import torch

    arr = (GemmProblem * len(problems))(*problems)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    check(_lib.lib().jc_gemm_group_device(device, precision_code(precision), arr, len(problems), s.cuda_stream))


def device_sync(device: int = 0) -> None:
    """Waits for the device and raises if a kernel's bounded wait gave up."""
    check(_lib.lib().jc_device_sync(device))
