"""ctypes binding of ``libjitcast_b200.so`` (the C ABI in ``include/jitcast_b200.h``).

The library is loaded from this package's directory; there is no fallback. If it is missing or
fails to load, every entry point raises ``JcUnavailable`` — the engine has no CPU path.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libjitcast_b200.so"

# jc_status
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED_SHAPE, ERR_OOM, ERR_CUDA, ERR_TIMEOUT, ERR_INTERNAL, ERR_NO_DEVICE = range(8)
STATUS_NAMES = ["OK", "INVALID_ARG", "UNSUPPORTED_SHAPE", "OOM", "CUDA", "TIMEOUT", "INTERNAL", "NO_DEVICE"]

# jc_precision
FP32, TF32, BF16, FP16 = 0, 1, 2, 3
PRECISIONS = {"fp32": FP32, "tf32": TF32, "bf16": BF16, "fp16": FP16}

# GEMM flags (tornado/Kernels.java:50-56, plus GELU)
BIAS, ACCUMULATE, SILU, TWIN_ONLY, RELU, GELU = 1, 2, 4, 8, 16, 32

# jc_time_attention_device flags
ATTN_CUDA_CORES = 1


class JcUnavailable(RuntimeError):
    """The native library is not built or cannot be loaded."""


class JcError(RuntimeError):
    """A non-OK jc_status, with the library's message."""

    def __init__(self, status: int, message: str):
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{name}: {message}")
        self.status = status
        self.message = message


class JcArgumentError(JcError, ValueError):
    """INVALID_ARG / UNSUPPORTED_SHAPE: the reference's IllegalArgumentException."""


_lib = None
_lock = threading.Lock()

c_int, c_ll, c_vp, c_char_p = ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_char_p
_fp = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes)
PROTOTYPES: dict[str, tuple] = {
    "jc_version": (c_char_p, []),
    "jc_last_error": (c_char_p, []),
    "jc_device_count": (c_int, []),
    "jc_linear": (c_int, [c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int]),
    "jc_linear_device": (c_int, [c_int, c_int, c_vp, c_ll, c_vp, c_ll, c_vp, c_vp, c_ll, c_int, c_int, c_int, c_int,
                                 c_vp]),
    "jc_linear_device_noalloc": (c_int, [c_int, c_int, c_vp, c_ll, c_vp, c_ll, c_vp, c_vp, c_ll, c_int, c_int, c_int,
                                         c_int, c_vp]),
    "jc_gemm_device": (c_int, [c_int, c_int, c_vp, c_vp, c_ll, c_vp, c_vp, c_ll, c_vp, c_vp, c_ll, c_int, c_int,
                               c_int, c_int, c_vp]),
    "jc_gemm_group_device": (c_int, [c_int, c_int, c_vp, c_int, c_vp]),
    "jc_device_sync": (c_int, [c_int]),
    "jc_device_wait_selftest": (c_int, [c_int, c_int]),
    "jc_shard_rows": (c_int, [c_int, c_vp, c_vp, c_int, c_vp]),
    "jc_timestral_prep_device": (c_int, [c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, ctypes.c_float, c_int, c_vp,
                                         c_vp]),
    "jc_chronos2_prep_device": (c_int, [c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, ctypes.c_float, c_int, c_vp,
                                        c_vp]),
    "jc_timestral_finish_device": (c_int, [c_int, c_int, c_int, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp]),
    "jc_chronos2_finish_device": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    "jc_time_attention_device": (c_int, [c_int, c_int, c_vp, c_ll, c_vp, c_ll, c_vp, c_ll, c_int, c_int, c_int, c_int,
                                         c_int, ctypes.c_float, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_int, c_vp]),
}


def declare(name: str, restype, argtypes) -> None:
    """Adds a prototype (used by the model modules for their entry points)."""
    PROTOTYPES[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype, fn.argtypes = restype, argtypes


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise JcUnavailable(f"{LIB_PATH} is not built (run python -m jitcast_b200.build)")
                try:
                    l = ctypes.CDLL(str(LIB_PATH))
                except OSError as e:
                    raise JcUnavailable(f"cannot load {LIB_PATH}: {e}") from e
                for name, (res, args) in PROTOTYPES.items():
                    fn = getattr(l, name)
                    fn.restype, fn.argtypes = res, args
                _lib = l
    return _lib


def last_error() -> str:
    return (lib().jc_last_error() or b"").decode()


def check(status: int) -> None:
    """Raises the reference-style exception for a non-OK status."""
    if status == OK:
        return
    msg = last_error()
    if status in (ERR_INVALID_ARG, ERR_UNSUPPORTED_SHAPE):
        raise JcArgumentError(status, msg)
    raise JcError(status, msg)


def precision_code(p) -> int:
    if isinstance(p, str):
        try:
            return PRECISIONS[p.lower()]
        except KeyError:
            raise ValueError(f"unknown precision {p!r}; expected one of {sorted(PRECISIONS)}") from None
    return int(p)
