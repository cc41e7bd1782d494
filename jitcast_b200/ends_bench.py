"""Times the host ends on the GPU (the scaler, token and finish kernels around a forward) through the C ABI.

    python -m jitcast_b200.ends_bench --family timestral --rows 8192 --context 4096 [--iters 5]
    python -m jitcast_b200.ends_bench --family chronos2 --rows 8192 --context 2048 [--iters 5]

A one-layer model of the family (d_model 128) keeps the forward between the kernels cheap; the ends do
not depend on the model's size, only on the window. Every call goes through ``jc_forecast_timestral`` /
``jc_forecast_chronos2`` with host buffers, eager (engine option ``profile``: CUDA events around every
launch). Prints one JSON line: per kernel its milliseconds per call (mean over ``--iters`` after
warm-up), its algorithmic bytes per call (each input byte read once, each output byte written once) and
the achieved GB/s.
"""

from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def _timestral(rows: int, context: int, horizon: int):
    from . import timestral as ts
    from . import workloads

    c = ts.TimestralConfig(patch_size=32, d_model=128, num_heads=2, mlp_hidden_dim=256, block_schedule=["time"],
                           quantile_knots=ts.default_knots(21), block_size=16, context_length=context).validate()
    eng = ts.TimestralEngine(c, ts.random_checkpoint(c, seed=0), precision="fp16")
    x = workloads.sinusoid_noise(rows, context, seed=0)
    lay = ts.BlockLayout.of(c, ts.BlockInput(x, np.ones_like(x, bool), np.arange(rows, dtype=np.int32), horizon))
    wi = ts.WindowInputs.of(c, lay)
    w, enc, hp, q = lay.encoder * c.patch_size, lay.encoder, horizon * c.patch_size, c.num_quantiles
    algo = {"prep.scaler": rows * (5 * w + 8 * enc + 1),
            "prep.tokens": rows * (5 * w + 8 * enc + 1 + 8 * w),
            "finish": rows * (2 * 4 * hp * q + 8)}
    return eng, (lambda: eng.forecast(wi)), algo


def _chronos2(rows: int, context: int, horizon: int):
    from . import chronos2 as c2
    from . import workloads

    c = c2.Chronos2Config(d_model=128, d_kv=64, d_ff=256, num_layers=1, num_heads=2,
                          quantiles=c2.default_quantiles(), context_length=context, patch_size=16,
                          max_output_patches=horizon, use_reg_token=True, use_arcsinh=True).validate()
    eng = c2.Chronos2Engine(c, c2.random_checkpoint(c, seed=0), precision="fp16")
    x = workloads.random_walk(rows, context, seed=0)
    lay = c2.ModelLayout.of(c, c2.ModelInput(x, np.arange(rows, dtype=np.int32), horizon))
    gs, ge = c2.group_ranges(lay.group)
    w, hp, q, ne = lay.context_patches * c.patch_size, horizon * c.patch_size, c.num_quantiles, \
        lay.context_patches + horizon
    algo = {"prep.norm": rows * (4 * w + 8),
            "prep.tokens": rows * (4 * (w + hp) + 8 + 12 * ne * c.patch_size),
            "finish": rows * (2 * 4 * q * hp + 8)}
    return eng, (lambda: eng.forecast(lay, gs, ge)), algo


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--family", default="timestral", choices=["timestral", "chronos2"])
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--context", type=int, default=None, help="steps (default 4096 Timestral, 2048 Chronos-2)")
    ap.add_argument("--horizon", type=int, default=None, help="patches (default 2 Timestral, 4 Chronos-2)")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)
    if args.family == "timestral":
        eng, call, algo = _timestral(args.rows, args.context or 4096, args.horizon or 2)
    else:
        eng, call, algo = _chronos2(args.rows, args.context or 2048, args.horizon or 4)
    with eng:
        for _ in range(args.warmup):
            call()
        eng.set_option("profile", 1)
        for _ in range(args.iters):
            call()
        prof = eng.profile()
    kernels = {}
    for name, bytes_ in algo.items():
        ms = prof[name]["ms"] / prof[name]["launches"]
        kernels[name] = {"ms": round(ms, 4), "bytes": bytes_, "gb_s": round(bytes_ / ms / 1e6, 1)}
    print(json.dumps({"family": args.family, "rows": args.rows, "context": args.context, "kernels": kernels}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
