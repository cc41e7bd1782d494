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


def shard_rows(group_start, group_end, parts: int):
    """``jc_shard_rows``: the first row of each of ``parts`` contiguous row ranges (and the row count last) that
    a multi-GPU forward gives its GPUs, no series split across two."""
    import numpy as np

    from ._lib import check

    gs = np.ascontiguousarray(group_start, np.int32)
    ge = np.ascontiguousarray(group_end, np.int32)
    cuts = np.empty(parts + 1, np.int32)
    check(lib().jc_shard_rows(len(gs), gs.ctypes.data, ge.ctypes.data, parts, cuts.ctypes.data))
    return cuts
