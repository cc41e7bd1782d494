"""The parity bars of the model tests, in one place.

The north star's bars, on every quantile level (max|a − e| / max|e| against the FP32 oracle):
  * JC_FP32, the FP32-accumulate mode: 1e-3 on the BASELINE configs;
  * JC_TF32: 1e-3; JC_BF16, the 16-bit tensor-core mode: 1e-2; JC_FP16 (same tensor rate, 10-bit mantissa): 1e-2.

A reduced-precision mode rounds every GEMM operand (weights and activations). Where that rounding alone moves
the reference's own arithmetic further than the bar, no implementation of the mode can meet the bar. The
reference's rule for its reduced-precision device paths covers this case: no further from the FP32 reference
than a reduced-precision run of the reference arithmetic (tirex2/tornado/TornadoForwardAccelTest.java:39-44,
GoldenData.nxaiGpuError). So a reduced-precision mode is held to the larger of its north-star bar and
FLOOR_FACTOR × that run's error (the "floor"): the oracle with every Ops.linear operand rounded to the mode's
format (``oracle.operand_format``), on the same inputs and weights. The factor leaves room for what the device
path does beyond rounding the GEMM operands: the tensor cores' truncating FP32 accumulation over a GEMM's whole K
in these modes (on the tiny TiRex-2 model in TF32 that alone takes the device to 1.55 × the floor) and the 16-bit
q, k, v and P of attention. JC_FP32 has no floor: its bar is the north star's.
"""

from __future__ import annotations

import oracle

NORTH_STAR = {"fp32": 1e-3, "tf32": 1e-3, "bf16": 1e-2, "fp16": 1e-2}
# the small test-only models keep the reference's FP32 device bar (TornadoForwardAccelTest.FP32_TOLERANCE)
TINY = {"fp32": 1e-4, "tf32": 1e-3, "bf16": 1e-2, "fp16": 1e-2}
FLOOR_FACTOR = 2.0


def bar(precision: str, reduced_run, err_of, base: dict | None = None) -> tuple[float, float | None]:
    """(bar, floor) for `precision`. ``reduced_run()`` runs the oracle forward that produced the expected output,
    and ``err_of(output)`` measures an output against the expected one; for the reduced-precision modes the run
    is repeated with the GEMM operands rounded to the mode's format and its error is the floor."""
    b = (base or NORTH_STAR)[precision]
    if precision == "fp32":
        return b, None
    with oracle.operand_format(precision):
        floor = float(err_of(reduced_run()))
    return max(b, FLOOR_FACTOR * floor), floor
