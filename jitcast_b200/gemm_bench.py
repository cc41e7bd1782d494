"""Times one tcgen05 GEMM shape through the C ABI (jc_gemm_device, operands resident in HBM).

    python -m jitcast_b200.gemm_bench --m 32768 --n 4096 --k 1024 --precision fp16 [--iters 20]
        [--epilogue plain|bias_silu|accumulate] [--cublas]

Prints one JSON line: milliseconds per call (CUDA events on the launching stream after warm-up),
achieved TFLOP/s, and the algorithmic bytes per call (A, W, C written, C read when accumulating).
``--cublas`` adds the same shape through cuBLAS as the reference calls it (torch.mm / torch.addmm with 16-bit
operands and an FP32 C) for comparison; ``--rounds R`` alternates the two R times (``--iters`` calls each) and
reports the median round of each, so that both see the same clocks; ``--single`` keeps the GEMM on
the single-CTA kernel (large shapes otherwise run on CTA pairs). BASELINE config 1 is
``--m 1024 --n 768 --k 256 --epilogue bias``.
"""

from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, required=True)
    ap.add_argument("--n", type=int, required=True)
    ap.add_argument("--k", type=int, required=True)
    ap.add_argument("--precision", default="fp16", choices=["fp16", "bf16", "tf32", "fp32"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--epilogue", default="plain", choices=["plain", "bias", "bias_silu", "accumulate"])
    ap.add_argument("--cublas", action="store_true")
    ap.add_argument("--rounds", type=int, default=1, help="alternate ours and cuBLAS this many times (median)")
    ap.add_argument("--single", action="store_true", help="keep the GEMM on the single-CTA kernel")
    args = ap.parse_args(argv)
    if args.single:
        import os

        os.environ["JC_GEMM_PAIR"] = "0"

    import torch

    from . import _lib

    L = _lib.lib()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    m, n, k = args.m, args.n, args.k
    prec = _lib.precision_code(args.precision)
    dt = {"fp16": torch.float16, "bf16": torch.bfloat16}.get(args.precision, torch.float32)
    g = torch.Generator(device=dev).manual_seed(0)
    kp = (k + 63) // 64 * 64
    a = torch.zeros(m, kp, device=dev, dtype=dt)
    w = torch.zeros(n, kp, device=dev, dtype=dt)
    a[:, :k] = torch.randn(m, k, device=dev, generator=g).to(dt)
    w[:, :k] = (torch.randn(n, k, device=dev, generator=g) / np.sqrt(k)).to(dt)
    a_lo = torch.zeros_like(a) if args.precision == "fp32" else None
    w_lo = torch.zeros_like(w) if args.precision == "fp32" else None
    bias = torch.zeros(n, device=dev)
    c = torch.zeros(m, n, device=dev)
    flags = {"plain": 0, "bias": _lib.BIAS, "bias_silu": _lib.BIAS | _lib.SILU, "accumulate": _lib.ACCUMULATE}[
        args.epilogue]
    stream = torch.cuda.Stream(dev)

    def call():
        st = L.jc_gemm_device(0, prec, a.data_ptr(), None if a_lo is None else a_lo.data_ptr(), kp, w.data_ptr(),
                              None if w_lo is None else w_lo.data_ptr(), kp, bias.data_ptr(), c.data_ptr(), n, m, n,
                              k, flags, stream.cuda_stream)
        _lib.check(st)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            for _ in range(args.iters):
                fn()
            e.record(stream)
            torch.cuda.synchronize()
        return s.elapsed_time(e) / args.iters

    cublas_fn = None
    if args.cublas and dt != torch.float32:
        # the reference's cuBLAS call: 16-bit operands, an FP32 C, β = 1 when accumulating (cublasGemmEx FP16 → FP32,
        # timestral/tornado/TimestralForward.java:483-492)
        cb = torch.zeros(m, n, device=dev, dtype=torch.float32)
        if flags & _lib.ACCUMULATE:
            cublas_fn = lambda: torch.addmm(cb, a[:, :k], w[:, :k].t(), out_dtype=torch.float32, out=cb)  # noqa: E731
        else:
            cublas_fn = lambda: torch.mm(a[:, :k], w[:, :k].t(), out_dtype=torch.float32, out=cb)  # noqa: E731
    ours_ms, cublas_ms = [], []
    for _ in range(max(1, args.rounds)):
        ours_ms.append(timed(call))
        _lib.check(L.jc_device_sync(0))
        if cublas_fn is not None:
            cublas_ms.append(timed(cublas_fn))
    ms = float(np.median(ours_ms))
    esz = 2 if dt != torch.float32 else 4
    bytes_ = (m * k + n * k) * esz * (2 if args.precision == "fp32" else 1) + m * n * 4 * (
        2 if flags & _lib.ACCUMULATE else 1)
    out = {"m": m, "n": n, "k": k, "precision": args.precision, "epilogue": args.epilogue, "ms": ms,
           "us": ms * 1e3, "tflops": 2.0 * m * n * k / (ms * 1e-3) / 1e12,
           "algorithmic_bytes": bytes_, "gbs": bytes_ / (ms * 1e-3) / 1e9}
    if cublas_ms:
        mc = float(np.median(cublas_ms))
        out["cublas_ms"] = mc
        out["cublas_tflops"] = 2.0 * m * n * k / (mc * 1e-3) / 1e12
        out["ours_over_cublas"] = mc / ms
    if args.rounds > 1:
        out["rounds"] = args.rounds
        out["ours_ms_rounds"] = ours_ms
        out["cublas_ms_rounds"] = cublas_ms
    print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
