"""Generates the golden fixtures for the GEMM path (run: python tests/golden/make_golden.py).

The reference's GEMM kernel tests (src/test/java/ai/beestream/jitcast/tornado/KernelsAccelTest.java:
57-149) draw their inputs from ``new java.util.Random(7)`` and compare every device GEMM with
``Ops.linear`` + SiLU/ReLU/accumulate (cpu/Ops.java:33-88). No JDK exists in this build
environment, so the expected outputs are computed here by an independent NumPy restatement of
Ops.linear's arithmetic — products rounded to double, summed sequentially in index order
(``np.cumsum`` accumulates left to right), the bias added in double, then rounded to float —
which is exactly what Java's strict IEEE double arithmetic produces. The C oracle must match these
bit for bit, and the CUDA GEMM within tolerance.

Fixture: ``kernels_gemm.npz`` with, per case, a / w / bias / c0 and the expected C per flag set.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import JavaRandom  # noqa: E402

BIAS, ACCUMULATE, SILU, RELU = 1, 2, 4, 16


def ops_linear(x, w, b):
    """Ops.linear in NumPy: sequential double accumulation, per output."""
    prod = x.astype(np.float64)[:, None, :] * w.astype(np.float64)[None, :, :]
    acc = np.cumsum(prod, axis=2)[:, :, -1]
    if b is not None:
        acc = acc + b.astype(np.float64)[None, :]
    return acc.astype(np.float32)


def silu(v):
    # in double, as Java promotes the float (Ops.java:68-70)
    return np.array([np.float32(float(x) / (1.0 + math.exp(-float(x)))) for x in v.ravel()], np.float32).reshape(v.shape)


def expected(a, w, bias, c0, flags):
    y = ops_linear(a, w, bias if flags & BIAS else None)
    if flags & SILU:
        y = silu(y)
    if flags & RELU:
        y = np.maximum(y, np.float32(0))
    if flags & ACCUMULATE:
        y = (y + c0).astype(np.float32)
    return y


def case(rnd, m, n, k, a_off, w_off, c_off, flags_list):
    """The draws of one KernelsAccelTest case, in its order: a, then w (+ bias), then c0."""
    a = rnd.gaussians(a_off + m * k, 1.0)
    w = rnd.gaussians(w_off + n * k + n, 0.2)
    c0 = rnd.gaussians(c_off + m * n, 1.0)
    A = a[a_off:a_off + m * k].reshape(m, k)
    W = w[w_off:w_off + n * k].reshape(n, k)
    B = w[w_off + n * k:w_off + n * k + n]
    C0 = c0[c_off:c_off + m * n].reshape(m, n)
    out = {"a": A, "w": W, "bias": B, "c0": C0, "flags": np.array(flags_list, np.int32)}
    for f in flags_list:
        out[f"exp_{f}"] = expected(A, W, B, C0, f)
    return out


def main():
    # One Random(7) per test method, as each JUnit test instance gets a fresh field initialiser.
    cases = {
        "every_flag": case(JavaRandom(7), 37, 45, 70, 0, 0, 0, [0, BIAS | SILU, BIAS | RELU, BIAS | ACCUMULATE]),
        "blocked": case(JavaRandom(7), 150, 200, 88, 5, 7, 3,
                        [0, BIAS | SILU, BIAS | RELU, BIAS | ACCUMULATE, ACCUMULATE]),
        "blocked_wide": case(JavaRandom(7), 150, 300, 88, 5, 7, 3,
                             [0, BIAS | SILU, BIAS | RELU, BIAS | ACCUMULATE, ACCUMULATE]),
    }
    flat = {f"{name}/{key}": val for name, d in cases.items() for key, val in d.items()}
    np.savez_compressed(HERE / "kernels_gemm.npz", **flat)
    print("wrote", HERE / "kernels_gemm.npz", sum(v.nbytes for v in flat.values()), "bytes")


if __name__ == "__main__":
    main()
