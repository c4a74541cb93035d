#!/usr/bin/env python
"""Benchmark of the B200 matvec path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one pass of the hot path over one batch of synthetic input: one
dequantize-and-dot matvec (batch 1) over a GGUF weight resident in HBM.

Workloads (default q4_0_11008x4096):
  q4_0_11008x4096      Q4_0 11008x4096 batch-1 matvec.  With N GPUs the weight is
                       (N*11008)x4096, row-sharded 11008 rows per GPU, and the y
                       slices are all-gathered over NCCL: weak scaling.
  q8_0_4096x4096       Q8_0 4096x4096 batch-1 matvec (weak scaling as above).
  f16_head_128000x2048 F16 128000x2048 LM-head matvec with the argmax fused.
  q4_0_32768x32768     Q4_0 32768x32768, row-sharded over N GPUs + NCCL all-gather
                       of y: strong scaling (fixed total matrix).
  q8_0_prefill_512x4096x14336
                       prompt-shaped batch: 512 token vectors through one Q8_0
                       14336x4096 weight (the tcgen05 GEMM), TFLOP/s; replicas
                       at N > 1.

Timing: W warm-up steps, then exactly K steps between a barrier +
cuda.synchronize on both sides, CUDA events on the launching stream, max over
ranks.  The K steps run as one CUDA graph (at N>1 with the NCCL all-gather of
each step inside it).  Weight copies rotate so the
rotating set exceeds 4x L2 (each step reads a weight that is not in L2).

`e2e` repeats the metric through the host entry point of the C ABI
(nedo_gpu_matvec: host x in, host y out, copies inside the timed region).
`cpu_baseline` times the reference's own CPU kernel (compiled from source into
oracle/_ref; the C restatement when that library is absent) on this host.
`--impl reference` times that same CPU kernel as the whole step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nedo.cpp_b200"))

import numpy as np  # noqa: E402

from nedo_gpu import blocks as B  # noqa: E402

METRIC = "Q8_0/Q4_0/F16 matvec HBM GB/s & % of B200 peak; prefill GEMM TFLOP/s @1-8 GPU"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1400.0

WORKLOADS = {
    "q4_0_11008x4096": dict(type=B.Q4_0, rows=11008, cols=4096, shard="weak", argmax=False),
    "q8_0_4096x4096": dict(type=B.Q8_0, rows=4096, cols=4096, shard="weak", argmax=False),
    "f16_head_128000x2048": dict(type=B.F16, rows=128000, cols=2048, shard="weak", argmax=True),
    "q4_0_32768x32768": dict(type=B.Q4_0, rows=32768, cols=32768, shard="strong", argmax=False),
    "q8_0_prefill_512x4096x14336": dict(type=B.Q8_0, rows=14336, cols=4096, shard="replica", argmax=False,
                                        batch=512),
}

# DRAM bytes (read + write) per launch of the dominant kernel, from ncu captures
# summarised under profiles/ (None where no capture exists for the workload).
NCU_TRAFFIC_BYTES = {
    "q4_0_11008x4096": 25_426_432,  # profiles/gemv_imma_q4_0_11008x4096.md
    "q8_0_4096x4096": 17_874_688,   # profiles/gemv_imma_q8_0_4096x4096.md
    "q8_0_prefill_512x4096x14336": 70_580_992,  # profiles/gemm_tc_q8_0_prefill_512x4096x14336.md
}


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def peaks(tensor=False):
    """(peak, source): HBM GB/s, or dense bf16 TFLOP/s for tensor-core workloads.
    The tensor figure is the sustained one: the timed region follows a 1 s soak
    and runs K back-to-back steps, the conditions of a long step under the power
    cap."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    key = "bf16_tflops_sustained" if tensor else "hbm_gbs"
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p[key]), f"measured (MEASURED_PEAKS.json {key})"
    except (OSError, KeyError, ValueError):
        return (FALLBACK_BF16_TFLOPS, "fallback 1.4 PFLOP/s sustained") if tensor else (FALLBACK_HBM_GBS,
                                                                                          "fallback 6.65 TB/s")


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def shard_rows(wl, world):
    if wl["shard"] in ("weak", "replica"):
        return wl["rows"], wl["rows"] * world
    assert wl["rows"] % world == 0
    return wl["rows"] // world, wl["rows"]


def algorithmic_bytes(type_, rows, cols):
    """W + x + y of one matvec (GGUF block bytes)."""
    return rows * B.row_bytes(type_, cols) + 4 * cols + 4 * rows


def batch_of(wl):
    return wl.get("batch", 1)


def work_of(wl, rows_total, batch=None):
    """(units, unit name, scale) of one step: bytes for matvecs, FLOPs for batches."""
    b = batch_of(wl) if batch is None else batch
    if batch_of(wl) > 1:
        return 2.0 * b * rows_total * wl["cols"], "TFLOP/s", 1e12
    return float(algorithmic_bytes(wl["type"], rows_total, wl["cols"])), "GB/s", 1e9


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_bench_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline
# The reference processes a prompt as one matvec per token (src/model.cpp:262-266);
# a batch workload's CPU sample is this many of them per call.
CPU_BATCH_SAMPLE = 8


def cpu_reference(type_, rows, cols, seed, nvec=1):
    """(callable, kind, cores) running the reference CPU kernel: `nvec` matvecs over one matrix."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    w = B.gen_weight(type_, rows, cols, seed)
    xs = [B.gen_x(cols, seed + k) for k in range(nvec)]
    if O.Reference.available():
        ref = O.Reference()
        cores = host_cores()
        ref.set_threads(cores)
        return (lambda: [ref.matvec(type_, rows, cols, w, x) for x in xs]), "reference", cores
    orc = O.Oracle()
    return (lambda: [orc.matvec(type_, rows, cols, w, x) for x in xs]), "port", 1


def time_cpu(fn, budget_s, max_calls):
    fn()
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (n == 0 or time.perf_counter() - t0 < budget_s):
        fn()
        n += 1
    return (time.perf_counter() - t0) / n, n


def cpu_baseline(wl, rows_total, budget_s=10.0):
    nvec = CPU_BATCH_SAMPLE if batch_of(wl) > 1 else 1
    fn, kind, cores = cpu_reference(wl["type"], rows_total, wl["cols"], seed=7, nvec=nvec)
    sec, n = time_cpu(fn, budget_s, 100000)
    units, unit, scale = work_of(wl, rows_total, batch=nvec)
    what = f"{B.TYPE_NAMES[wl['type']]} {rows_total}x{wl['cols']} matvecs"
    if nvec > 1:
        what = f"{nvec}-token samples of the {batch_of(wl)}-token batch ({what}, one per token)"
    return {"value": round(units / sec / scale, 4), "unit": unit, "cores": cores, "kind": kind,
            "sample": f"{n} x {what} ({sec * 1e3:.3f} ms each, {n * sec:.1f} s)"}


def run_reference_arm(args, wl, world, rank):
    if rank != 0:
        return
    _, rows_total = shard_rows(wl, world)
    nvec = CPU_BATCH_SAMPLE if batch_of(wl) > 1 else 1
    fn, kind, cores = cpu_reference(wl["type"], rows_total, wl["cols"], seed=7, nvec=nvec)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    sec = (time.perf_counter() - t0) / args.steps
    units, unit, scale = work_of(wl, rows_total, batch=nvec)
    gbs = units / sec / scale
    line = {
        "metric": METRIC, "value": round(gbs, 4), "unit": unit, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 4), "higher_is_better": True,
        "scaling": "strong" if wl["shard"] == "strong" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded GGUF blocks)",
        "config": workload_config(args.workload, wl, world),
        "cpu_baseline": {"value": round(gbs, 4), "unit": unit, "cores": cores, "kind": kind,
                         "sample": f"each step {nvec} full {B.TYPE_NAMES[wl['type']]} {rows_total}x{wl['cols']} "
                                   f"matvec{'s (a sample of the batch, one per token)' if nvec > 1 else ''}"},
        "e2e": {"value": round(gbs, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(name, wl, world):
    rows, rows_total = shard_rows(wl, world)
    t = B.TYPE_NAMES[wl["type"]]
    desc = f"{t} matvec {rows_total}x{wl['cols']} batch {batch_of(wl)}"
    if batch_of(wl) > 1:
        desc = (f"{t} {wl['rows']}x{wl['cols']} weight x {batch_of(wl)} token vectors "
                f"(prefill GEMM, M={batch_of(wl)} K={wl['cols']} N={wl['rows']})")
        if world > 1:
            desc += f", {world} independent replicas"
    elif world > 1:
        desc += f", row-sharded {rows} rows per GPU + NCCL all-gather of y"
    if wl["argmax"]:
        desc += ", argmax fused"
    return {"workload": name, "description": desc, "type": t, "rows_total": rows_total, "rows_per_gpu": rows,
            "cols": wl["cols"], "batch": batch_of(wl),
            "parallelism": ("replicas" if wl["shard"] == "replica" else f"rowshard{world}") if world > 1 else "single"}


# ------------------------------------------------------------------ GPU arm
def make_weights(torch, type_, rows, cols, copies, seed, device):
    """`copies` independent seeded weights [copies, rows*row_bytes] (uint8) on device."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nb = cols // 32
    if type_ == B.F16:
        w = (torch.randn((copies, rows, cols), generator=g, device=device) * 0.02).half()
        return w.view(torch.uint8).reshape(copies, -1)
    bb = B.BLOCK_BYTES[type_]
    blk = torch.empty((copies, rows, nb, bb), dtype=torch.uint8, device=device)
    if type_ == B.Q8_0:
        q = torch.randint(-127, 128, (copies, rows, nb, 32), generator=g, device=device, dtype=torch.int16)
        blk[..., 2:] = q.to(torch.int8).view(torch.uint8)
        d = (torch.randn((copies, rows, nb), generator=g, device=device).abs() * (0.02 / 127.0)).half()
    else:
        blk[..., 2:] = torch.randint(0, 256, (copies, rows, nb, 16), generator=g, device=device,
                                     dtype=torch.int16).to(torch.uint8)
        d = (torch.randn((copies, rows, nb), generator=g, device=device).abs() * (0.02 / 8.0)).half()
    blk[..., 0:2] = d.contiguous().view(torch.uint8).reshape(copies, rows, nb, 2)
    return blk.reshape(copies, -1)


def run_gpu_arm(args, wl, world, rank, local_rank):
    import torch
    import torch.distributed as dist

    import nedo_gpu
    from nedo_gpu.shard import ShardedMatvec

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    lib = nedo_gpu.load()
    # Programmatic dependent launch: each matvec starts streaming its weight
    # while the previous launch drains (x is read only after it completed).
    lib.set_pdl(True)
    t, cols = wl["type"], wl["cols"]
    rows, rows_total = shard_rows(wl, world)
    rb = B.row_bytes(t, cols)
    shard_bytes = rows * rb
    copies = max(1, math.ceil(4 * L2_BYTES / shard_bytes))
    w = make_weights(torch, t, rows, cols, copies, seed=1000 + rank, device=device)
    gx = torch.Generator(device=device)
    gx.manual_seed(7)
    nb = batch_of(wl)
    x = torch.randn((nb, cols) if nb > 1 else cols, generator=gx, device=device, dtype=torch.float32)
    y = torch.empty((nb, rows) if nb > 1 else rows, dtype=torch.float32, device=device)
    y_full = torch.empty(rows_total, dtype=torch.float32, device=device) if world > 1 and nb == 1 else y
    idx = torch.zeros(1, dtype=torch.int64, device=device)
    val = torch.zeros(1, dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device=device)
    plan = lib.plan_info(t, rows, cols, nb)

    def launch(k, s):
        wp = w[k % copies].data_ptr()
        if wl["argmax"]:
            lib.matvec_argmax_dev(t, rows, cols, wp, x.data_ptr(), y.data_ptr(), idx.data_ptr(), val.data_ptr(), s)
        else:
            lib.matvec_dev(t, rows, cols, wp, x.data_ptr(), y.data_ptr(), nb, s)

    # N > 1: this rank's rows, then the NCCL all-gather of the y slices
    # (replica workloads run independently on every GPU: no collective)
    sm = ShardedMatvec(t, rows_total, cols) if world > 1 and wl["shard"] != "replica" else None

    def step(k):
        if sm is None:
            launch(k, stream.cuda_stream)
        else:
            sm.run(lambda xv, yl: launch(k, stream.cuda_stream), x, y, y_full)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        tt = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    with torch.cuda.stream(stream):
        for k in range(max(3, args.warmup)):
            step(k)
    torch.cuda.synchronize()
    lib.status(stream.cuda_stream)

    # Kernel-only CUDA graph of K launches (the roofline's launch duration and, at
    # N=1, the whole step).
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for k in range(args.steps):
            launch(k, torch.cuda.current_stream().cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    # N > 1: the whole step (matvec + NCCL all-gather) as one graph of K steps;
    # every rank captures the same collectives in the same order
    step_graph = None
    if world > 1:
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(step_graph, stream=stream):
            for k in range(args.steps):
                step(k)
        step_graph.replay()
        torch.cuda.synchronize()
        barrier()

    sampler = ClockSampler(local_rank)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    while time.perf_counter() < soak_end:  # clocks under load before the timed region
        graph.replay()
        torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        if world == 1:
            graph.replay()
        else:
            step_graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    region_ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = sampler.stop()

    # kernel-only timing (all ranks, for the roofline)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        k0.record(stream)
        graph.replay()
        k1.record(stream)
    torch.cuda.synchronize()
    kernel_ms = max_over_ranks(k0.elapsed_time(k1)) / args.steps
    lib.status(stream.cuda_stream)
    del graph
    del step_graph  # holds NCCL calls: released before the process group goes

    units_total, unit, scale = work_of(wl, rows_total)  # whole job, all ranks
    ms_per_step = region_ms / args.steps
    value = units_total / (ms_per_step * 1e-3) / scale

    # ---- end to end through the C ABI host entry point
    e2e = e2e_measure(args, lib, torch, dist, wl, w, copies, rows, rows_total, world, rank, device, stream)

    tensor = nb > 1
    peak, peak_kind = peaks(tensor)
    per_launch, _, _ = work_of(wl, rows)
    achieved = per_launch / (kernel_ms * 1e-3) / scale
    traffic = NCU_TRAFFIC_BYTES.get(args.workload) if world == 1 else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
        "scaling": "strong" if wl["shard"] == "strong" else "weak", "vs_baseline": None,
        # block dots on the int8 tensor pipe (exact int32) for the IMMA plan; fp16
        # operands with fp32 accumulation on tcgen05 for batches; fp32 FMA otherwise
        "dtype": {4: "int8", 5: "f16"}.get(plan.get("path"), "f32"),
        "data": "synthetic (seeded GGUF blocks, torch.Generator on device)",
        "config": dict(workload_config(args.workload, wl, world),
                       l2=f"{copies} rotating weight copies ({copies * shard_bytes / 2**20:.0f} MiB per GPU, "
                          f"> 4x L2)", graph="K steps (matvec" + (" + NCCL all-gather" if world > 1 else "")
                          + ") captured as one CUDA graph",
                       pdl=True, plan=plan),
        "roofline": {"bound": "tensor" if tensor else "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_kind,
                     "launch_us": round(kernel_ms * 1e3, 3),
                     ("flops_per_step" if tensor else "bytes_per_launch"): per_launch},
        "e2e": e2e,
        # one matvec kernel per step (argmax fused into it); batches: x -> fp16, then the GEMM
        "gpu_launches": args.steps * (2 if plan.get("path") == 5 else 1),
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, rows_total)
    if rank == 0:
        print(json.dumps(line), flush=True)


def e2e_measure(args, lib, torch, dist, wl, w, copies, rows, rows_total, world, rank, device, stream):
    t, cols = wl["type"], wl["cols"]
    nb = batch_of(wl)
    if nb > 1:
        # a prompt-sized batch end to end: pinned host x -> device, the batched
        # matvec (x -> fp16 + tcgen05 GEMM), y -> pinned host, every step
        x_pin = torch.from_numpy(np.random.default_rng(7).standard_normal((nb, cols), dtype=np.float32)).pin_memory()
        y_pin = torch.empty((nb, rows), dtype=torch.float32).pin_memory()
        xd = torch.empty((nb, cols), dtype=torch.float32, device=device)
        yd = torch.empty((nb, rows), dtype=torch.float32, device=device)

        def one(k):
            with torch.cuda.stream(stream):
                xd.copy_(x_pin, non_blocking=True)
                lib.matvec_dev(t, rows, cols, w[k % copies].data_ptr(), xd.data_ptr(), yd.data_ptr(), nb,
                               stream.cuda_stream)
                y_pin.copy_(yd, non_blocking=True)
            stream.synchronize()

        for k in range(3):
            one(k)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for k in range(args.steps):
            one(k)
        sec = time.perf_counter() - t0
        if world > 1:
            tt = torch.tensor([sec], dtype=torch.float64, device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            sec = float(tt.item())
        sec /= args.steps
        units, unit, scale = work_of(wl, rows_total)
        return {"value": round(units / sec / scale, 2), "unit": unit, "h2d_bytes_per_step": 4 * nb * cols,
                "d2h_bytes_per_step": 4 * nb * rows,
                "path": "pinned H2D + nedo_gpu_matvec_dev(batch) + D2H", "ms_per_step": round(sec * 1e3, 4)}
    x_host = np.random.default_rng(7).standard_normal(cols, dtype=np.float32)
    n_host = min(copies, 8) if world == 1 else 1
    if world == 1:
        hosts = [w[i].cpu().numpy() for i in range(n_host)]
        for h in hosts:  # residency: first call uploads
            lib.matvec(t, rows, cols, h, x_host)
        t0 = time.perf_counter()
        for k in range(args.steps):
            y_host = lib.matvec(t, rows, cols, hosts[k % n_host], x_host)
        sec = (time.perf_counter() - t0) / args.steps
        assert y_host.shape == (rows,)
        for h in hosts:
            lib.weight_evict(h)
        bytes_total = algorithmic_bytes(t, rows_total, cols)
        return {"value": round(bytes_total / sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * cols,
                "d2h_bytes_per_step": 4 * rows, "path": "nedo_gpu_matvec (host pointers, resident weight)",
                "ms_per_step": round(sec * 1e3, 4)}
    # N > 1: pinned host x -> device, shard matvec, NCCL all-gather, full y -> host
    x_pin = torch.from_numpy(x_host).pin_memory()
    y_pin = torch.empty(rows_total, dtype=torch.float32).pin_memory()
    xd = torch.empty(cols, dtype=torch.float32, device=device)
    y = torch.empty(rows, dtype=torch.float32, device=device)
    y_full = torch.empty(rows_total, dtype=torch.float32, device=device)

    from nedo_gpu.shard import ShardedMatvec

    sm = ShardedMatvec(t, rows_total, cols)

    def one(k):
        with torch.cuda.stream(stream):
            xd.copy_(x_pin, non_blocking=True)
            sm.run(lambda xv, yl: lib.matvec_dev(t, rows, cols, w[k % copies].data_ptr(), xv.data_ptr(),
                                                 yl.data_ptr(), 1, stream.cuda_stream), xd, y, y_full)
            y_pin.copy_(y_full, non_blocking=True)
        stream.synchronize()

    for k in range(3):
        one(k)
    dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        one(k)
    sec = time.perf_counter() - t0
    tt = torch.tensor([sec], dtype=torch.float64, device=device)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    sec = float(tt.item()) / args.steps
    bytes_total = algorithmic_bytes(t, rows_total, cols)
    return {"value": round(bytes_total / sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * cols,
            "d2h_bytes_per_step": 4 * rows_total, "path": "pinned H2D + nedo_gpu_matvec_dev + NCCL all-gather + D2H",
            "ms_per_step": round(sec * 1e3, 4)}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="q4_0_11008x4096", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    wl = WORKLOADS[args.workload]

    if args.impl == "reference":
        run_reference_arm(args, wl, world, rank)
        return

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_gpu_arm(args, wl, world, rank, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
