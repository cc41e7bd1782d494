"""jitcast_b200 — the B200-native forward-pass GEMM engine behind jitCast's forward interfaces.

The compute runs in ``libjitcast_b200.so`` (hand-written tcgen05/TMA kernels for sm_100a, C ABI
in ``include/jitcast_b200.h``). This package is the host-side mirror of the reference's
interfaces over that ABI: ``ops`` (Kernels.gemm / Ops.linear) and one module per model family.
"""

from ._lib import BF16, FP32, TF32, JcArgumentError, JcError, JcUnavailable, lib  # noqa: F401
from . import ops  # noqa: F401

__version__ = "0.1.0"


def version() -> str:
    return lib().jc_version().decode()
