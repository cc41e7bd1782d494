"""ORACLE — test infrastructure only.

ctypes bindings to the C restatement of the reference's FP32 CPU operators and forwards
(``oracle/*.c``), plus a restatement of ``java.util.Random`` so tests can draw the same inputs
the reference's own tests draw (``new Random(7).nextGaussian()`` in KernelsAccelTest).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this package, and only as the checker. The product path (``jitcast_b200``) never does.
"""

from __future__ import annotations

import contextlib
import ctypes
import math
import os
from pathlib import Path

import numpy as np

from . import build as _build

_lib: ctypes.CDLL | None = None

BIAS, ACCUMULATE, SILU, RELU, GELU = 1, 2, 4, 16, 32

_F = ctypes.POINTER(ctypes.c_float)


def lib() -> ctypes.CDLL:
    """The oracle's shared library, built on first use."""
    global _lib
    if _lib is None:
        path = _build.OUT if _build.OUT.exists() else _build.build()
        _lib = ctypes.CDLL(str(path))
        _lib.jco_linear.argtypes = [_F, ctypes.c_int, _F, _F, ctypes.c_int, ctypes.c_int, _F, ctypes.c_int]
        _lib.jco_rmsnorm.argtypes = [_F, ctypes.c_int, ctypes.c_int, _F, ctypes.c_float, _F]
        _lib.jco_gemm.argtypes = [_F, _F, _F, _F, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int]
        _lib.jco_set_operand_format.argtypes = [ctypes.c_int]
        _lib.jco_operand_format.restype = ctypes.c_int
        _lib.jco_round_operand.argtypes = [ctypes.c_float, ctypes.c_int]
        _lib.jco_round_operand.restype = ctypes.c_float
        _lib.jco_silu.argtypes = [ctypes.c_float]
        _lib.jco_silu.restype = ctypes.c_float
        for name, fn in _extra_bindings():
            fn(_lib)
    return _lib


_EXTRA: list = []


def _extra_bindings():
    return list(_EXTRA)


def register(name: str):
    """Registers a function that declares more ctypes prototypes on the oracle library."""

    def deco(fn):
        _EXTRA.append((name, fn))
        if _lib is not None:
            fn(_lib)
        return fn

    return deco


def fptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


# jco_set_operand_format codes: a reduced-precision run of the reference arithmetic
OPERAND_FORMATS = {"fp32": 0, "tf32": 1, "bf16": 2, "fp16": 3}


@contextlib.contextmanager
def operand_format(name: str):
    """Within the block every oracle GEMM (``Ops.linear``) rounds its operands to ``name`` ("tf32", "bf16",
    "fp16"; "fp32" = the reference's arithmetic) before its double accumulation: the reduced-precision run of
    the reference arithmetic that the reference holds its reduced-precision device paths to
    (tirex2/tornado/TornadoForwardAccelTest.java:39-44, GoldenData.nxaiGpuError)."""
    lib().jco_set_operand_format(OPERAND_FORMATS[name])
    try:
        yield
    finally:
        lib().jco_set_operand_format(0)


def threads() -> int:
    return int(os.environ.get("JCO_THREADS", os.cpu_count() or 1))


def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None, nthreads: int | None = None) -> np.ndarray:
    """``Ops.linear`` (cpu/Ops.java:33-51): x [rows, in], w [out, in], b [out] or None."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    b = None if b is None else np.ascontiguousarray(b, np.float32)
    rows, k = x.shape
    n = w.shape[0]
    y = np.empty((rows, n), np.float32)
    lib().jco_linear(fptr(x), rows, fptr(w), fptr(b), k, n, fptr(y), nthreads or threads())
    return y


def gemm(a, w, bias, c0, flags: int, nthreads: int | None = None) -> np.ndarray:
    """Kernels.gemm's expected output as KernelsAccelTest composes it (linear, SiLU, ReLU, += C)."""
    a = np.ascontiguousarray(a, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    m, k = a.shape
    n = w.shape[0]
    c = np.zeros((m, n), np.float32) if c0 is None else np.array(c0, np.float32, copy=True).reshape(m, n)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().jco_gemm(fptr(a), fptr(w), fptr(b), fptr(c), m, n, k, flags, nthreads or threads())
    return c


def rmsnorm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    y = np.empty_like(x)
    lib().jco_rmsnorm(fptr(x), rows, cols, fptr(None if w is None else np.ascontiguousarray(w, np.float32)),
                      eps, fptr(y))
    return y


def rel_max_err(actual: np.ndarray, expected: np.ndarray) -> float:
    """The reference's check: max|a − e| / max(max|e|, 1e-6) (KernelHarness.java:104-117,
    TimestralGolden.java:125-140). NaN in `actual` where `expected` is finite gives inf."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    if np.any(np.isnan(a) & ~np.isnan(e)):
        return math.inf
    scale = max(float(np.max(np.abs(e))) if e.size else 0.0, 1e-6)
    return float(np.max(np.abs(a - e))) / scale if e.size else 0.0


class JavaRandom:
    """``java.util.Random``: the 48-bit LCG and the polar-method ``nextGaussian`` of its
    published specification, so tests draw the inputs of ``new Random(seed)`` exactly."""

    _MULT = 0x5DEECE66D
    _MASK = (1 << 48) - 1

    def __init__(self, seed: int):
        self._seed = (seed ^ self._MULT) & self._MASK
        self._next_gaussian: float | None = None

    def _next(self, bits: int) -> int:
        self._seed = (self._seed * self._MULT + 0xB) & self._MASK
        v = self._seed >> (48 - bits)
        if v >= 1 << 31:  # Java's (int) cast
            v -= 1 << 32
        return v

    def next_double(self) -> float:
        hi = self._next(26) & ((1 << 26) - 1)
        lo = self._next(27) & ((1 << 27) - 1)
        return ((hi << 27) + lo) * (1.0 / (1 << 53))

    def next_gaussian(self) -> float:
        if self._next_gaussian is not None:
            g, self._next_gaussian = self._next_gaussian, None
            return g
        while True:
            v1 = 2 * self.next_double() - 1
            v2 = 2 * self.next_double() - 1
            s = v1 * v1 + v2 * v2
            if 0 < s < 1:
                break
        mul = math.sqrt(-2 * math.log(s) / s)
        self._next_gaussian = v2 * mul
        return v1 * mul

    def gaussians(self, n: int, scale: float) -> np.ndarray:
        """``(float) nextGaussian() * scale`` n times, as KernelsAccelTest.random builds its inputs."""
        g = np.array([self.next_gaussian() for _ in range(n)], np.float64).astype(np.float32)
        return (g * np.float32(scale)).astype(np.float32)


__all__ = ["lib", "linear", "gemm", "rmsnorm", "rel_max_err", "JavaRandom", "register", "fptr", "threads",
           "BIAS", "ACCUMULATE", "SILU", "RELU", "GELU", "Path"]
