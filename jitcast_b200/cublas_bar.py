"""The bar to beat on B200: the reference's default CUDA path at the models' shapes, against this engine.

    python -m jitcast_b200.cublas_bar [--series 8192] [--precision fp16|bf16] [--iters 3]
    python -m jitcast_b200.cublas_bar --peaks      # cuBLAS BF16 and TF32 dense peaks, burst and sustained

The reference's CUDA default (timestral/tornado/TimestralForward.java:404-499, ``GemmMode.CUBLAS_FP16``) runs
every linear layer as cuBLAS ``cublasGemmExFP16FP32``: FP16 operands, an FP32 C (β = 1 to accumulate), plus
separate passes over HBM around it: ``toHalf`` of the GEMM input, ``biasFill`` before a biased GEMM, ``biasSilu``
after a SiLU one, ``rope`` on q and k, ``gate`` (att · σ(gate)) and ``swiGlu``. Per stage of one config-5
chunk (the config-3 model over 8,192 series, the chunk ``bench.py`` times) this prints:

* ``cublas_ms``: the stage's GEMMs through torch at identical (M, K, N) — ``torch.mm(..., out_dtype=float32)``
  or ``torch.addmm(c, ..., out_dtype=float32)`` for β = 1, i.e. cuBLAS GemmEx FP16 → FP32 as the reference
  calls it — timed with CUDA events;
* ``passes_ms``: the stage's unfused passes at their HBM floor (bytes read + written ÷ the measured HBM copy
  bandwidth), a lower bound on what those kernels cost;
* ``bar_ms`` = cublas_ms + passes_ms, and ``ours_ms``: the same stage in this engine (its tcgen05 GEMMs with the
  epilogues fused), from a profiled forward of the same chunk (CUDA events around every launch).

Each line is one JSON object; a final ``total`` line sums the stages.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


def hbm_gbs() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"])
    return 6650.0  # the profiling recipe's fallback


def timed(fn, iters: int, warmup: int = 2) -> float:
    """Milliseconds per call, CUDA events on the current stream after warm-up."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def stages(series: int, d: int = 1024, f: int = 4096, P: int = 32, Q: int = 21, enc: int = 128, h: int = 2,
           layers: int = 16):
    """The config-3 model's linear stages for one chunk: (name, repeat, [GEMM (M, K, N, beta)], pass bytes).
    Pass bytes follow TimestralForward's CUBLAS_FP16 plan: toHalf reads 4 and writes 2 bytes per input element,
    biasFill writes C (reads it too before an accumulating GEMM), biasSilu reads and writes C, rope reads and
    writes q and k, gate reads att and gate and writes att, swiGlu reads the 2F-wide C and writes F."""
    T = series * (enc + h)
    E = series * enc
    D = series * h
    PQ = P * Q
    th = lambda m, k: 6 * m * k  # noqa: E731
    return [
        ("gemm.embed", 1, [(E, 2 * P, f, 0), (E, f, d, 1), (E, 2 * P, d, 1)],
         th(E, 2 * P) + 8 * E * f + th(E, f) + 4 * E * d + th(E, 2 * P) + 8 * E * d),
        ("gemm.qkvg", layers, [(T, d, 3 * d, 0), (T, d, d, 0)],
         th(T, d) + 16 * T * d + th(T, d) + 12 * T * d),
        ("gemm.wo", layers, [(T, d, d, 1)], th(T, d)),
        ("gemm.w12", layers, [(T, d, 2 * f, 0)], th(T, d) + (8 * f + 4 * f) * T),
        ("gemm.w3", layers, [(T, f, d, 1)], th(T, f)),
        ("gemm.head", 1, [(D, d, f, 0), (D, f, PQ, 1), (D, d, PQ, 1)],
         th(D, d) + 8 * D * f + th(D, f) + 4 * D * PQ + th(D, d) + 8 * D * PQ),
    ]


def cublas_stage(gemms, dt, iters: int) -> float:
    """cuBLAS time of one instance of a stage's GEMMs (FP16/BF16 operands, FP32 C)."""
    import torch

    dev = torch.device("cuda", 0)
    ms = 0.0
    for m, k, n, beta in gemms:
        a = torch.randn(m, k, device=dev, dtype=dt)
        w = torch.randn(n, k, device=dev, dtype=dt) / np.sqrt(k)
        c = torch.zeros(m, n, device=dev, dtype=torch.float32)
        if beta:
            fn = lambda: torch.addmm(c, a, w.t(), out_dtype=torch.float32, out=c)  # noqa: E731
        else:
            fn = lambda: torch.mm(a, w.t(), out_dtype=torch.float32, out=c)  # noqa: E731
        ms += timed(fn, iters)
        del a, w, c
        torch.cuda.empty_cache()
    return ms


def ours_profile(series: int, precision: str) -> dict:
    """Per-stage CUDA-event times of one profiled forecast of a config-5 chunk through this engine."""
    import torch

    from . import timestral as ts
    from . import workloads

    dev = torch.device("cuda", 0)
    c = ts.config3()
    w = ts.random_checkpoint(c, seed=0)
    x = workloads.sinusoid_noise(series, 4096, seed=0)
    b = ts.BlockInput(x, np.ones_like(x, bool), np.arange(series, dtype=np.int32), 2)
    stream = torch.cuda.Stream(dev)
    with ts.TimestralEngine(c, w, precision=precision) as eng:
        dw = ts.DeviceWindow(ts.WindowInputs.of(c, ts.BlockLayout.of(c, b)), dev)
        out = torch.empty(dw.out_shape(c), device=dev)
        for _ in range(2):
            dw.forecast(eng, out, stream)
        eng.sync()
        eng.set_option("profile", 1)
        dw.forecast(eng, out, stream)
        eng.sync()
        prof = eng.profile()
    return prof


def peaks(seconds: float = 4.0) -> list[dict]:
    """cuBLAS dense peaks at 8192³ through torch: BF16 and TF32 (allow_tf32), best of 10 (burst) and back to
    back for `seconds` (sustained, under the power cap)."""
    import torch

    dev = torch.device("cuda", 0)
    n = 8192
    out = []
    for name, dt, tf32 in (("bf16", torch.bfloat16, False), ("tf32", torch.float32, True)):
        torch.backends.cuda.matmul.allow_tf32 = tf32
        a = torch.randn(n, n, device=dev, dtype=dt)
        b = torch.randn(n, n, device=dev, dtype=dt)
        c = torch.empty(n, n, device=dev, dtype=dt)
        fn = lambda: torch.matmul(a, b, out=c)  # noqa: E731
        best = min(timed(fn, 1, warmup=3 if i == 0 else 0) for i in range(10))
        calls, t0 = 0, time.perf_counter()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        while time.perf_counter() - t0 < seconds:
            for _ in range(20):
                fn()
            calls += 20
            torch.cuda.synchronize()
        e.record()
        torch.cuda.synchronize()
        sus = s.elapsed_time(e) / calls
        flops = 2.0 * n ** 3
        out.append({"peak": name, "burst_tflops": flops / (best * 1e-3) / 1e12,
                    "sustained_tflops": flops / (sus * 1e-3) / 1e12, "n": n, "sustained_s": seconds})
        del a, b, c
        torch.cuda.empty_cache()
    torch.backends.cuda.matmul.allow_tf32 = False
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--series", type=int, default=8192)
    ap.add_argument("--precision", default="fp16", choices=["fp16", "bf16"])
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--peaks", action="store_true", help="measure the cuBLAS BF16 and TF32 dense peaks instead")
    args = ap.parse_args(argv)
    import torch

    torch.cuda.set_device(0)
    if args.peaks:
        for line in peaks():
            print(json.dumps(line), flush=True)
        return 0
    dt = torch.float16 if args.precision == "fp16" else torch.bfloat16
    gbs = hbm_gbs()
    prof = ours_profile(args.series, args.precision)
    tot = {"cublas_ms": 0.0, "passes_ms": 0.0, "bar_ms": 0.0, "ours_ms": 0.0, "flops": 0.0}
    for name, rep, gemms, pass_bytes in stages(args.series):
        cub = rep * cublas_stage(gemms, dt, args.iters)
        passes = rep * pass_bytes / (gbs * 1e9) * 1e3
        flops = rep * sum(2.0 * m * k * n for m, k, n, _ in gemms)
        ours = prof.get(name, {}).get("ms", float("nan"))
        line = {"stage": name, "launches_per_stage": len(gemms), "layers": rep, "cublas_ms": cub,
                "cublas_tflops": flops / (cub * 1e-3) / 1e12, "passes_ms": passes, "pass_bytes": rep * pass_bytes,
                "bar_ms": cub + passes, "ours_ms": ours, "ours_tflops": flops / (ours * 1e-3) / 1e12,
                "speedup_vs_bar": (cub + passes) / ours}
        print(json.dumps(line), flush=True)
        for k_, v in (("cublas_ms", cub), ("passes_ms", passes), ("bar_ms", cub + passes), ("ours_ms", ours),
                      ("flops", flops)):
            tot[k_] += v
    print(json.dumps({"stage": "total", "series": args.series, "precision": args.precision, "hbm_gbs": gbs, **tot,
                      "cublas_tflops": tot["flops"] / (tot["cublas_ms"] * 1e-3) / 1e12,
                      "ours_tflops": tot["flops"] / (tot["ours_ms"] * 1e-3) / 1e12,
                      "speedup_vs_bar": tot["bar_ms"] / tot["ours_ms"]}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
