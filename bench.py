"""Benchmark: Timestral-style forward passes on the B200 engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one forward pass of the whole box-scale batch (65,536 series by default, sharded evenly
across the N ranks; each rank runs its series in chunks of up to 8,192 through one CUDA graph per
chunk shape). Prints one JSON line on rank 0:

* ``value``   series/s of the whole job, inputs already in HBM (jc_forward_timestral_device), device
              time by CUDA events, max over ranks;
* ``e2e``     the same metric through the host C-ABI call (jc_forward_timestral with host buffers,
              host↔device copies inside the timed region);
* ``roofline`` the dominant kernel (the tcgen05 GEMM) from a profiled forward on rank 0: algorithmic
              FLOPs per launch ÷ its CUDA-event time, against the measured BF16 peak;
* ``cpu_baseline`` the oracle (a C restatement of the reference's FP32 CPU forward; the reference is
              Java and no JDK exists here) on a bounded sample, rank 0 at N = 1.

``--impl reference`` times that CPU forward on the host cores instead (rank 0; other ranks exit).
``--workload config2|config4`` times BASELINE configs 2 (Chronos-2, 256 series) and 4 (TiRex-2, 512 series) on one
GPU with the same rules (a step is one forward of the config's batch).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "series forecasts/sec (Timestral-style config-3 model, box-scale batch of config 5)"
GEMM_BYTES_PER_LAUNCH_1024 = 1.736e9
UNIT = "series/s"


def rank_chunks(series: int, chunk: int, world: int, rank: int) -> list[tuple[int, int]]:
    """The (first series, count) of every forward call of one rank: the batch split evenly over the ranks, each
    share in chunks. Chunks are seeded by their first series, so every N runs the same series."""
    per_rank = series // world
    first = rank * per_rank
    return [(c0, min(chunk, first + per_rank - c0)) for c0 in range(first, first + per_rank, chunk)]


def max_over_ranks(v: float, world: int, device) -> float:
    """The largest of every rank's v (the whole job's time is its slowest rank's)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--series", type=int, default=65536, help="series per step, whole job")
    ap.add_argument("--chunk", type=int, default=8192, help="series per forward call")
    ap.add_argument("--precision", default="fp16", choices=["fp16", "bf16", "tf32", "fp32"])
    ap.add_argument("--cpu-series", type=int, default=2, help="series in the CPU baseline sample")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-engine", action="store_true",
                    help="skip the multi-GPU engine measurement (N > 1: one process, one engine over all N GPUs)")
    ap.add_argument("--workload", default="config5", choices=["config5", "config2", "config4"],
                    help="config5 (default: the headline box-scale Timestral batch), config2 (Chronos-2, 256 "
                         "series) or config4 (TiRex-2, 512 series), one GPU")
    return ap.parse_args()


def workload_config(args, world):
    return {"workload": "config5: Timestral-style decoder (d 1024, 16 layers, 16 heads, SwiGLU 4096, patch 32, "
                        "128 context tokens + 2 decoder tokens, 21 quantiles), random-init weights",
            "series_per_step": args.series, "series_per_gpu": args.series // world, "chunk_series": args.chunk,
            "context": 4096, "horizon_patches": 2, "tokens_per_series": 130, "precision": args.precision,
            "parallelism": f"series-sharded x{world}, no collective",
            "path": "value: jc_forecast_timestral_device on each chunk's window, observed flags and layout resident "
                    "in HBM (BlockPrep.of, the forward and BlockPrep.finish on the GPU); e2e: jc_forecast_timestral "
                    "from pinned host buffers, copies timed; BlockLayout.of before the timed region",
            "l2": "no flush: every forward's working set (GBs) is far larger than the 126 MB L2"}


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_sample(cfg, weights, series: int):
    """The oracle's CPU forward on `series` series of the same workload; returns (series/s, threads)."""
    from jitcast_b200 import timestral as ts
    from jitcast_b200 import workloads
    from oracle import timestral as ots

    x = workloads.sinusoid_noise(series, 4096, seed=12345)
    b = ts.BlockInput(x, np.ones_like(x, bool), np.arange(series, dtype=np.int32), 2)
    model = ots.Model(cfg, weights)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    model.predict_block(b, nthreads=threads)
    dt = time.perf_counter() - t0
    return series / dt, threads


def reference_arm(args, rank, world):
    """The reference's CPU forward (C restatement) on the host cores, for the same metric."""
    if rank != 0:
        return 0
    from jitcast_b200 import timestral as ts

    cfg = ts.config3()
    weights = ts.random_checkpoint(cfg, seed=0)
    for _ in range(args.warmup):
        cpu_sample(cfg, weights, 1)
    vals, threads = [], 1
    for _ in range(args.steps):
        v, threads = cpu_sample(cfg, weights, args.cpu_series)
        vals.append(v)
    value = statistics.median(vals)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * args.cpu_series / value, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64-accumulate f32", "data": "synthetic",
            "config": workload_config(args, world), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{args.cpu_series} series per step of the config-5 workload, "
                                       "C restatement of CpuTimestral.predictBlock (no JDK on this image)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# GEMM FLOPs per series of one forward (2·M·K·N summed over the model's linear layers at the configs' shapes:
# Chronos-2 config 2 with 128 context + [REG] + 4 future tokens, TiRex-2 config 4 with headwise gates)
WORKLOAD_GEMM_FLOPS = {"config2": 30.82e9, "config4": 5.02e9}


def engine_profile(L, handle):
    import ctypes

    from jitcast_b200 import _lib

    cap = 32
    names = (ctypes.c_char_p * cap)()
    ms = (ctypes.c_double * cap)()
    launches = (ctypes.c_longlong * cap)()
    flops = (ctypes.c_double * cap)()
    n = ctypes.c_int()
    _lib.check(L.jc_engine_profile(handle, 0, names, ms, launches, flops, cap, ctypes.byref(n)))
    return {names[i].decode(): {"ms": ms[i], "launches": launches[i], "flops": flops[i]} for i in range(n.value)}


def pinned(a: np.ndarray) -> np.ndarray:
    """A copy of ``a`` in pinned (page-locked) host memory, C-contiguous."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()


def pinned_empty(shape: tuple) -> np.ndarray:
    """An uninitialised float32 array in pinned host memory."""
    import torch

    return torch.empty(shape, dtype=torch.float32, pin_memory=True).numpy()


def engine_multi_gpu(args, cfg, weights, world: int) -> dict:
    """The library's own multi-GPU path, as a Java caller reaches it: ONE TimestralEngine over devices 0..N-1 and
    jc_forecast_timestral on host buffers (the block's rows sharded over the GPUs on series boundaries, one host
    thread per GPU, each shard's finished quantiles copied into one pinned caller buffer; SeriesWindows.split,
    host/SeriesWindows.java:37-56). Each call carries N chunks of ``--chunk`` series (every GPU runs a chunk, as
    the per-process bench does); a step is the whole batch. Wall-clock time of the calls (each returns after its
    gather), copies included."""
    from jitcast_b200 import timestral as ts
    from jitcast_b200 import workloads

    engine = ts.TimestralEngine(cfg, weights, devices=tuple(range(world)), precision=args.precision)
    per_call = args.chunk * world
    calls = []
    for c0 in range(0, args.series, per_call):
        n = min(per_call, args.series - c0)
        # the same chunk-seeded series as the per-process bench
        x = np.concatenate([workloads.sinusoid_noise(min(args.chunk, c0 + n - s0), 4096, seed=s0)
                            for s0 in range(c0, c0 + n, args.chunk)])
        b = ts.BlockInput(x, np.ones_like(x, bool), np.arange(n, dtype=np.int32), 2)
        wi = ts.WindowInputs.of(cfg, ts.BlockLayout.of(cfg, b))
        lp = dataclasses.replace(wi.layout, **{k: pinned(getattr(wi.layout, k)) for k in ts.DeviceWindow.FIELDS})
        hp = dataclasses.replace(wi, layout=lp, window=pinned(wi.window), observed=pinned(wi.observed))
        calls.append((hp, pinned_empty((n, 2 * cfg.patch_size, cfg.num_quantiles))))
    for hp, qp in calls:  # warm-up: plans and graphs on every GPU
        engine.forecast(hp, out=qp)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for hp, qp in calls:
            engine.forecast(hp, out=qp)
    dt = (time.perf_counter() - t0) / args.steps
    engine.close()
    return {"value": args.series / dt, "unit": UNIT, "n_gpus": world, "ms_per_step": 1000.0 * dt,
            "calls_per_step": len(calls), "series_per_call": per_call,
            "path": "one process: jc_forecast_timestral on a TimestralEngine over devices 0..N-1 (rows sharded on "
                    "series boundaries, one host thread per GPU, quantiles gathered into one pinned caller buffer); "
                    "host buffers, copies timed, wall clock"}


def workload_bench(args, world):
    """Configs 2 and 4 on one GPU, with config 5's timing rules: a step is one forward of the config's batch."""
    import ctypes

    import torch

    from jitcast_b200 import _lib
    from jitcast_b200 import workloads

    if world > 1:
        print(json.dumps({"error": f"--workload {args.workload} runs on one GPU"}))
        return 2
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L = _lib.lib()
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    if args.workload == "config2":
        from jitcast_b200 import chronos2 as c2

        cfg = c2.config2()
        batch = 256
        weights = c2.random_checkpoint(cfg, seed=0)
        engine = c2.Chronos2Engine(cfg, weights, precision=args.precision)
        x = workloads.random_walk(batch, 2048, seed=0)
        inp = c2.ModelInput(x, np.arange(batch, dtype=np.int32), 4)
        lay = c2.ModelLayout.of(cfg, inp)
        prep = c2.ModelPrep.of(cfg, lay)
        gs, ge = c2.group_ranges(np.asarray(inp.group))
        d = {"tok": t(np.asarray(prep.tokens, np.float32)), "live": t(np.asarray(lay.live, np.int32)),
             "gs": t(gs), "ge": t(ge)}
        out = torch.empty(lay.rows * lay.output_patches, cfg.num_quantiles * cfg.patch_size, device=dev)
        blk = c2.Block(lay.rows, lay.context_patches, lay.output_patches, d["tok"].data_ptr(), d["live"].data_ptr(),
                       d["gs"].data_ptr(), d["ge"].data_ptr())
        device_fwd = lambda: L.jc_forward_chronos2_device(engine.handle, 0, ctypes.byref(blk), out.data_ptr(),
                                                          stream.cuda_stream)
        # e2e from pinned host buffers (jc_forecast_chronos2): the window, future covariates, live flags and group
        # ranges in; ModelPrep.of, the encoder and ModelPrep.finish on the GPU; the finished quantiles out
        pwin, pfut = pinned(np.asarray(lay.window, np.float32)), pinned(np.asarray(lay.future, np.float32))
        plive, pgs, pge = pinned(np.asarray(lay.live, np.int32)), pinned(gs), pinned(ge)
        lay_p = dataclasses.replace(lay, window=pwin, future=pfut, live=plive)
        q_p = pinned_empty((lay.rows, cfg.num_quantiles, lay.output_patches * cfg.patch_size))
        host_fwd = lambda: engine.forecast(lay_p, pgs, pge, out=q_p)
        h2d = pwin.nbytes + pfut.nbytes + plive.nbytes + pgs.nbytes + pge.nbytes
        d2h = q_p.nbytes
        desc = ("config2: Chronos-2-style T5 encoder (d 768, 12 layers, 12 heads, d_ff 3072 ReLU, patch 16, 128 "
                "context + [REG] + 4 future tokens, 21 quantiles), random-init weights")
        data = "synthetic random walks x_t = x_{t-1} + N(0,1), seed 0"
    else:
        from jitcast_b200 import tirex2 as tx

        cfg = tx.config4()
        batch = 512
        weights = tx.random_checkpoint(cfg, seed=0)
        engine = tx.TiRex2Engine(cfg, weights, precision=args.precision)
        x = workloads.ar2(batch, cfg.padded_length, seed=0)
        x[:, cfg.context_len:] = np.nan
        b = tx.ModelBatch(x, np.arange(batch, dtype=np.float32), np.ones(batch, bool))
        di = tx.DeviceInputs.of(cfg, b)
        st = di.st
        d = {k: t(v) for k, v in dict(x=di.x, present=di.present, known=st.known, kept=st.kept, gs=st.group_start,
                                     ge=st.group_end, kt=st.kept_target).items()}
        out = torch.empty(batch, cfg.num_quantiles, cfg.padded_length, device=dev)
        blk = tx.Batch(batch, d["x"].data_ptr(), d["present"].data_ptr(), len(st.known), d["known"].data_ptr(),
                       len(st.kept), d["kept"].data_ptr(), d["gs"].data_ptr(), d["ge"].data_ptr(), d["kt"].data_ptr())
        device_fwd = lambda: L.jc_forward_tirex2_device(engine.handle, 0, ctypes.byref(blk), out.data_ptr(),
                                                        stream.cuda_stream)
        # e2e from pinned host buffers: values and presence flags in, quantiles out
        di_p = dataclasses.replace(di, x=pinned(di.x), present=pinned(di.present))
        out_p = pinned_empty(tuple(out.shape))
        host_fwd = lambda: engine.forward_inputs(di_p, out=out_p)
        h2d = di_p.x.nbytes + di_p.present.nbytes
        d2h = out_p.nbytes
        desc = ("config4: TiRex-style xLSTM stack (d 512, 12 blocks, sLSTM at 3, 7, 11, 4 heads, patch 32, 64 "
                "patches, 9 quantiles, input/output FF 2048), random-init weights")
        data = "synthetic AR(2) phi1 0.6 phi2 0.3 sigma 1, 200-step burn-in, seed 0"
    for _ in range(max(args.warmup, 3)):
        _lib.check(device_fwd())
    torch.cuda.synchronize()
    engine.sync()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        time.sleep(0.3)  # nvidia-smi's first sample
        start.record(stream)
        for _ in range(args.steps):
            _lib.check(device_fwd())
        stop.record(stream)
        torch.cuda.synchronize()
        # a timed region shorter than the sampling period gets its clock samples from the same forward repeated
        # (untimed) until a second has passed
        t_end = time.perf_counter() + max(0.0, 1.0 - start.elapsed_time(stop) / 1e3)
        while time.perf_counter() < t_end:
            _lib.check(device_fwd())
            torch.cuda.synchronize()
    engine.sync()
    ms = start.elapsed_time(stop) / args.steps
    host_fwd()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_fwd()
    e2e_s = (time.perf_counter() - t0) / args.steps
    engine.set_option("profile", 1)
    _lib.check(device_fwd())
    torch.cuda.synchronize()
    prof = engine_profile(L, engine.handle)
    ends_prof = {}
    if args.workload == "config2":  # the host ends on the GPU of one end-to-end forecast, timed the same way
        host_fwd()
        ends_prof = {k: v for k, v in engine_profile(L, engine.handle).items() if k.startswith(("prep", "finish"))}
    engine.set_option("profile", 0)
    gemms = {k: v for k, v in prof.items() if k.startswith("gemm")}
    g = {f: sum(v[f] for v in gemms.values()) for f in ("ms", "launches", "flops")}
    pk, pk_kind = peaks()
    peak_tf = pk.get("bf16_tflops_sustained", 1400.0)
    achieved = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] else 0.0
    line = {"metric": f"series forecasts/sec ({args.workload})", "value": batch / (ms / 1000.0), "unit": UNIT,
            "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.precision,
            "data": data, "config": {"workload": desc, "series_per_step": batch, "precision": args.precision,
                                     "l2": "no flush: every forward's working set is far larger than the L2"},
            "e2e": {"value": batch / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": None,
                         "kernel": "gemm_pair_kernel / gemm_tc_kernel (tcgen05, all linear layers)",
                         "peak_kind": f"{pk_kind} bf16 dense, sustained",
                         "gemm_time_share": g["ms"] / sum(v["ms"] for v in prof.values()),
                         "gemm_flops_per_series": WORKLOAD_GEMM_FLOPS[args.workload]},
            "cpu_baseline": None, "clocks": clocks.summary(),
            "gpu_launches": sum(v["launches"] for v in prof.values()) * args.steps,
            "kernel_profile": {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                                   **({"tflops": round(v["flops"] / v["ms"] / 1e9, 1)} if v["flops"] else {})}
                               for k, v in prof.items()},
            "host_ends_profile": {k: {"ms": round(v["ms"], 3), "launches": v["launches"]} for k, v in ends_prof.items()}}
    print(json.dumps(line), flush=True)
    engine.close()
    return 0


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.workload != "config5":
        return workload_bench(args, world)

    import datetime

    import torch
    import torch.distributed as dist

    from jitcast_b200 import timestral as ts
    from jitcast_b200 import workloads

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    cfg = ts.config3()
    weights = ts.random_checkpoint(cfg, seed=0)
    engine = ts.TimestralEngine(cfg, weights, devices=(local,), precision=args.precision)

    per_rank = args.series // world
    chunks = []
    win_in = []  # each chunk's window and layout (host arrays), for the end-to-end forecast
    lay_fields = ts.DeviceWindow.FIELDS
    for c0, n in rank_chunks(args.series, args.chunk, world, rank):
        x = workloads.sinusoid_noise(n, 4096, seed=c0)  # chunk-seeded: the same series for every N
        b = ts.BlockInput(x, np.ones_like(x, bool), np.arange(n, dtype=np.int32), 2)
        wi = ts.WindowInputs.of(cfg, ts.BlockLayout.of(cfg, b))
        win_in.append(wi)
        # resident in HBM: the window, its observed flags and the layout; the GPU runs BlockPrep.of, the forward
        # and BlockPrep.finish (jc_forecast_timestral_device)
        dw = ts.DeviceWindow(wi, dev)
        out = torch.empty(dw.out_shape(cfg), device=dev)
        chunks.append((wi, dw, out, n))
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)

    def device_step():
        for _, dw, out, _ in chunks:
            dw.forecast(engine, out, stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def over_ranks(v: float) -> float:
        return max_over_ranks(v, world, dev)

    for _ in range(max(args.warmup, 3)):
        device_step()
    torch.cuda.synchronize()
    engine.sync()

    barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            device_step()
        stop.record(stream)
        torch.cuda.synchronize()
    engine.sync()
    barrier()
    ms = over_ranks(start.elapsed_time(stop) / args.steps)
    value = args.series / (ms / 1000.0)

    # end to end through the host C ABI (jc_forecast_timestral): each chunk's window, observed flags and layout
    # from pinned host buffers, BlockPrep's scaler and tokens, the forward and BlockPrep.finish on the GPU, the
    # finished quantiles back into pinned host buffers, copies timed (the layout itself is built before)
    fields = lay_fields
    host_chunks = []
    for wi, (_, _, _, n) in zip(win_in, chunks):
        lp = dataclasses.replace(wi.layout, **{k: pinned(getattr(wi.layout, k)) for k in fields})
        hp = dataclasses.replace(wi, layout=lp, window=pinned(wi.window), observed=pinned(wi.observed))
        qp = pinned_empty((n, 2 * cfg.patch_size, cfg.num_quantiles))
        host_chunks.append((hp, qp, n))
    for hp, qp, _ in host_chunks[:1]:
        engine.forecast(hp, out=qp)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    h2d = d2h = 0
    for _ in range(args.steps):
        for hp, qp, n in host_chunks:
            engine.forecast(hp, out=qp)
            h2d += hp.window.nbytes + hp.observed.nbytes + sum(getattr(hp.layout, k).nbytes for k in fields)
            d2h += qp.nbytes
    e2e_s = over_ranks((time.perf_counter() - t0) / args.steps)
    barrier()

    # kernel-class timings of one profiled forecast (eager, CUDA events around every launch)
    engine.set_option("profile", 1)
    _, dw0, out0, _ = chunks[0]
    dw0.forecast(engine, out0, stream)
    torch.cuda.synchronize()
    prof = engine.profile()
    engine.set_option("profile", 0)
    ends_prof = {k: v for k, v in prof.items() if k.startswith(("prep", "finish"))}
    launches_per_forward = sum(v["launches"] for v in prof.values()) + 3  # + the 3 index-rebasing kernels
    gemms = {k: v for k, v in prof.items() if k.startswith("gemm")}
    g = {f: sum(v[f] for v in gemms.values()) for f in ("ms", "launches", "flops")}
    gemm_ms = g["ms"] / g["launches"]
    gemm_flops = g["flops"] / g["launches"]
    pk, pk_kind = peaks()
    peak_tf = pk.get("bf16_tflops_sustained", 1400.0)
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12
    # DRAM bytes (read + written) per GEMM launch, from one ncu capture of every GEMM launch of a 1,024-series
    # forward (dram__bytes_read.sum + dram__bytes_write.sum: 114.6 GB over 66 launches = 1.736 GB each, FP16
    # operands), scaled by the chunk's series: the activations are all but a few MB of it and grow with the rows.
    traffic = GEMM_BYTES_PER_LAUNCH_1024 * min(args.chunk, per_rank) / 1024.0 if args.precision == "fp16" else None

    # the library's own multi-GPU engine (N > 1): every rank frees its GPU, rank 0 drives all N from one process
    # while the others wait on a host-side (gloo) barrier, so no collective kernel waits on a GPU meanwhile
    engine_line = None
    n_chunks = len(chunks)
    if world > 1 and not args.no_engine:
        engine.close()
        chunks.clear()  # the device windows and outputs
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=1200))
        if rank == 0:
            engine_line = engine_multi_gpu(args, cfg, weights, world)
        dist.barrier(group=host_group)
    if rank != 0:
        engine.close()
        if world > 1:
            dist.destroy_process_group()
        return 0
    cpu = None
    if world == 1 and not args.no_cpu:
        v, threads = cpu_sample(cfg, weights, args.cpu_series)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{args.cpu_series} series of the config-5 workload through the C restatement of "
                         "CpuTimestral.predictBlock (FP32, double accumulation; no JDK on this image)"}
    total_gemm_share = g["ms"] / sum(v["ms"] for v in prof.values())
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
            "config": workload_config(args, world),
            # whole-job bytes: every rank moves the same share
            "e2e": {"value": args.series / e2e_s, "unit": UNIT, "h2d_bytes_per_step": world * h2d // args.steps,
                    "d2h_bytes_per_step": world * d2h // args.steps},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": traffic,
                         "kernel": "gemm_pair_kernel / gemm_tc_kernel (tcgen05, all linear layers)",
                         "peak_kind": f"{pk_kind} bf16 dense, sustained",
                         "gemm_time_share": total_gemm_share},
            "cpu_baseline": cpu, "clocks": clocks.summary(),
            "gpu_launches": launches_per_forward * n_chunks * args.steps,
            "kernel_profile": {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                                   **({"tflops": round(v["flops"] / v["ms"] / 1e9, 1)} if v["flops"] else {})}
                               for k, v in prof.items()},
            "host_ends_profile": {k: {"ms": round(v["ms"], 3), "launches": v["launches"]} for k, v in ends_prof.items()}}
    if engine_line is not None:
        line["engine_multi_gpu"] = engine_line
    print(json.dumps(line), flush=True)
    engine.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
