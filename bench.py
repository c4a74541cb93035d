#!/usr/bin/env python
"""Benchmark of the B200 matvec path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one pass of the hot path over one batch of synthetic input: one
dequantize-and-dot matvec (batch 1) over a GGUF weight resident in HBM.

Workloads (default q4_0_11008x4096):
  q4_0_11008x4096      Q4_0 11008x4096 batch-1 matvec.  With N GPUs every GPU
                       streams its own 11008x4096 row block (rows are independent:
                       no exchange on the data path): weak scaling.
  q8_0_4096x4096       Q8_0 4096x4096 batch-1 matvec (weak scaling as above).
  f16_head_128000x2048 F16 128000x2048 LM-head matvec with the argmax fused
                       (weak scaling as above).
  q4_0_32768x32768     Q4_0 32768x32768, row-sharded over N GPUs with the y slices
                       all-gathered: the matvec kernel stores its rows on every
                       peer over NVLink (NCCL where that kernel does not take the
                       shape): strong scaling (fixed total matrix).
  q8_0_prefill_512x4096x14336
                       prompt-shaped batch: 512 token vectors through one Q8_0
                       14336x4096 weight (the tcgen05 GEMM), TFLOP/s; replicas
                       at N > 1.
  decode_sweep_24x1536_b1, _b8, _b32
                       every matvec of a synthetic 24-layer decoder (d_model 1536:
                       q/k/v/o 1536x1536, gate/up 4096x1536, down 1536x4096, Q8_0)
                       plus an F16 64000x1536 head, for 1, 8 or 32 tokens per step
                       (the head takes the argmax at batch 1); GB/s with each
                       weight counted once per step, per-matrix GB/s in the line.

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
    "q4_0_11008x4096": dict(type=B.Q4_0, rows=11008, cols=4096, shard="replica", argmax=False),
    "q8_0_4096x4096": dict(type=B.Q8_0, rows=4096, cols=4096, shard="replica", argmax=False),
    "f16_head_128000x2048": dict(type=B.F16, rows=128000, cols=2048, shard="replica", argmax=True),
    "q4_0_32768x32768": dict(type=B.Q4_0, rows=32768, cols=32768, shard="strong", argmax=False),
    "q8_0_prefill_512x4096x14336": dict(type=B.Q8_0, rows=14336, cols=4096, shard="replica", argmax=False,
                                        batch=512),
}
for _b in (1, 8, 32):
    WORKLOADS[f"decode_sweep_24x1536_b{_b}"] = dict(kind="sweep", type=B.Q8_0, layers=24, d=1536, ff=4096,
                                                    head=64000, batch=_b, shard="replica", argmax=_b == 1,
                                                    rows=1536, cols=1536)


def sweep_matrices(wl):
    """(name, type, rows, cols) of one decode step, in call order."""
    d, ff = wl["d"], wl["ff"]
    layer = [("q", d, d), ("k", d, d), ("v", d, d), ("o", d, d), ("gate", ff, d), ("up", ff, d), ("down", d, ff)]
    mats = [(f"{n}{li}", wl["type"], r, c) for li in range(wl["layers"]) for n, r, c in layer]
    return mats + [("head", B.F16, wl["head"], d)]


def sweep_bytes(wl, batch):
    """Algorithmic bytes of one step: every weight once, x and y per token."""
    return sum(r * B.row_bytes(t, c) + batch * 4 * (r + c) for _, t, r, c in sweep_matrices(wl))

# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu
# capture of the same workload (dram__bytes_read.sum + dram__bytes_write.sum);
# absent where no capture exists for the workload.
NCU_TRAFFIC_BYTES = {
    "q4_0_11008x4096": 25_444_352,
    "q8_0_4096x4096": 17_893_632,
    "q4_0_32768x32768": 609_625_344,
    "f16_head_128000x2048": 527_622_400,
    "q8_0_prefill_512x4096x14336": 70_827_776,
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
    if wl.get("kind") == "sweep":
        cb = sweep_cpu(wl, budget_s=min(20.0, 0.05 * args.steps + 2.0))
        line = {"metric": METRIC, "value": cb["value"], "unit": "GB/s", "impl": "reference", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF blocks)",
                "config": {"workload": args.workload, "batch": batch_of(wl)},
                "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                            "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
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
    elif world > 1 and wl["shard"] == "replica":
        desc += f", {world} independent {rows}-row blocks (one per GPU, no exchange)"
    elif world > 1:
        desc += f", row-sharded {rows} rows per GPU + all-gather of y"
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
    from nedo_gpu.shard import FusedShardedMatvec, ShardedMatvec

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

    # N > 1: this rank's rows, then every rank gets all of y -- fused into the
    # int8 tensor-pipe kernel as NVLink peer stores where it takes the shape,
    # else an NCCL all-gather (replica workloads run independently: no collective)
    sm = fm = None
    collective = None
    if world > 1 and wl["shard"] != "replica":
        if plan.get("path") == 4 and nb == 1:
            fm = FusedShardedMatvec(lib, t, rows_total, cols, device)
            collective = "fused: rows stored on every peer over NVLink by the matvec kernel + completion wait"
        else:
            sm = ShardedMatvec(t, rows_total, cols)
            collective = "NCCL all-gather of the y slices"

    def step(k):
        if fm is not None:
            fm.run(w[k % copies].data_ptr(), x.data_ptr(), torch.cuda.current_stream().cuda_stream)
        elif sm is not None:
            sm.run(lambda xv, yl: launch(k, stream.cuda_stream), x, y, y_full)
        else:
            launch(k, stream.cuda_stream)

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
    # N > 1: the whole step (matvec + all-gather) as one graph of K steps (K
    # rounded to even: the fused path alternates two gathered buffers); every
    # rank captures the same collectives in the same order
    step_graph = None
    if world > 1:
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(step_graph, stream=stream):
            for k in range(args.steps + (args.steps & 1)):
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
    if world > 1:
        region_ms *= args.steps / (args.steps + (args.steps & 1))
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
    e2e = e2e_measure(args, lib, torch, dist, wl, w, copies, rows, rows_total, world, rank, device, stream, fm)

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
                       pdl=True, plan=plan, **({"collective": collective} if collective else {})),
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


def run_sweep_arm(args, wl, world, rank, local_rank):
    """Decode sweep: every matvec of one decoder step (plus the head) per step,
    all weights resident (918 MB: more than 4x L2, so each step reads HBM)."""
    import torch
    import torch.distributed as dist

    import nedo_gpu

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    lib = nedo_gpu.load()
    lib.set_pdl(True)
    nb = batch_of(wl)
    mats = sweep_matrices(wl)
    ws = [make_weights(torch, t, r, c, 1, seed=2000 + 7 * i + rank, device=device)[0]
          for i, (_, t, r, c) in enumerate(mats)]
    d, ff = wl["d"], wl["ff"]
    g = torch.Generator(device=device)
    g.manual_seed(7)
    xd = torch.randn((nb, d), generator=g, device=device)
    xf = torch.randn((nb, ff), generator=g, device=device)
    yd = torch.empty((nb, d), device=device)
    yf = torch.empty((nb, ff), device=device)
    logits = torch.empty((nb, wl["head"]), device=device)
    idx = torch.zeros(1, dtype=torch.int64, device=device)
    val = torch.zeros(1, dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device=device)

    def one(i, s):
        name, t, r, c = mats[i]
        x = xf if c == ff else xd
        y = logits if name == "head" else (yf if r == ff else yd)
        if name == "head" and wl["argmax"]:
            lib.matvec_argmax_dev(t, r, c, ws[i].data_ptr(), x.data_ptr(), y.data_ptr(), idx.data_ptr(),
                                  val.data_ptr(), s)
        else:
            lib.matvec_dev(t, r, c, ws[i].data_ptr(), x.data_ptr(), y.data_ptr(), nb, s)

    def step(s):
        for i in range(len(mats)):
            one(i, s)

    def max_over_ranks(v):
        if world == 1:
            return v
        tt = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step(stream.cuda_stream)
    torch.cuda.synchronize()
    lib.status(stream.cuda_stream)
    steps = max(1, min(args.steps, 50))  # about 1 ms per step
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps):
            step(torch.cuda.current_stream().cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    while time.perf_counter() < soak_end:
        graph.replay()
        torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_per_step = max_over_ranks(ev0.elapsed_time(ev1)) / steps
    clocks = sampler.stop()
    del graph
    lib.status(stream.cuda_stream)

    # per matrix kind: the 24 layers' launches of one kind (or the head) as one graph
    kinds = {}
    for i, (name, t, r, c) in enumerate(mats):
        kinds.setdefault(name.rstrip("0123456789"), []).append(i)
    per_kind = {}
    for kind, ids in kinds.items():
        kg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kg, stream=stream):
            for _ in range(3):
                for i in ids:
                    one(i, torch.cuda.current_stream().cuda_stream)
        kg.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            kg.replay()
            b.record(stream)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / (3 * len(ids))
        _, t, r, c = mats[ids[0]]
        byts = r * B.row_bytes(t, c) + nb * 4 * (r + c)
        per_kind[f"{kind} {B.TYPE_NAMES[t]} {r}x{c}"] = {"us": round(us, 3), "GB/s": round(byts / us / 1e3, 1),
                                                       "path": lib.plan_info(t, r, c, nb)["path"]}
        del kg

    units_total = sweep_bytes(wl, nb) * world
    value = units_total / (ms_per_step * 1e-3) / 1e9
    peak, peak_kind = peaks()
    launches = sum(nb if (lib.plan_info(t, r, c, nb)["path"] in (3, 4) and nb > 1) else
                   (2 if lib.plan_info(t, r, c, nb)["path"] == 5 else 1) for _, t, r, c in mats)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic (seeded GGUF blocks, torch.Generator on device)",
        "config": {"workload": args.workload,
                   "description": f"{wl['layers']}-layer d_model {d} decoder step: {len(mats) - 1} Q8_0 matvecs + "
                                  f"F16 {wl['head']}x{d} head, {nb} token(s) per step",
                   "batch": nb, "weight_bytes_per_step": sum(r * B.row_bytes(t, c) for _, t, r, c in mats),
                   "parallelism": "replicas" if world > 1 else "single",
                   "l2": "918 MB of weights, all resident: each step streams them from HBM (> 4x L2)",
                   "graph": f"{steps} steps of {len(mats)} matvecs captured as one CUDA graph", "pdl": True,
                   "per_matrix": per_kind},
        "roofline": {"bound": "hbm", "achieved": round(value / world, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(value / world / peak, 4), "traffic": None, "peak_source": peak_kind,
                     "launch_us": round(ms_per_step * 1e3, 3), "bytes_per_step": sweep_bytes(wl, nb)},
        "e2e": None,
        "gpu_launches": steps * launches,
        "clocks": clocks,
    }
    # end to end: pinned host x in, the step, pinned logits out
    x_pin = torch.randn((nb, d)).pin_memory()
    l_pin = torch.empty((nb, wl["head"])).pin_memory()
    reps = 5
    with torch.cuda.stream(stream):
        xd.copy_(x_pin, non_blocking=True)
        step(stream.cuda_stream)
        l_pin.copy_(logits, non_blocking=True)
    stream.synchronize()
    t0 = time.perf_counter()
    for _ in range(reps):
        with torch.cuda.stream(stream):
            xd.copy_(x_pin, non_blocking=True)
            step(stream.cuda_stream)
            l_pin.copy_(logits, non_blocking=True)
        stream.synchronize()
    sec = max_over_ranks(time.perf_counter() - t0) / reps
    line["e2e"] = {"value": round(units_total / sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * nb * d,
                   "d2h_bytes_per_step": 4 * nb * wl["head"], "path": "pinned H2D + 169 nedo_gpu_matvec_dev + D2H",
                   "ms_per_step": round(sec * 1e3, 4)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = sweep_cpu(wl, budget_s=10.0)
    if rank == 0:
        print(json.dumps(line), flush=True)


def sweep_cpu(wl, budget_s=10.0):
    """The reference CPU kernels over one token of the sweep (all 169 matvecs)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    mats = sweep_matrices(wl)
    data = [(t, r, c, B.gen_weight(t, r, c, 3000 + i), B.gen_x(c, 3000 + i)) for i, (_, t, r, c) in enumerate(mats)]
    if O.Reference.available():
        ref, kind, cores = O.Reference(), "reference", host_cores()
        ref.set_threads(cores)
    else:
        ref, kind, cores = O.Oracle(), "port", 1

    def fn():
        for t, r, c, w, x in data:
            ref.matvec(t, r, c, w, x)

    sec, n = time_cpu(fn, budget_s, 1000)
    units = sweep_bytes(wl, 1)
    return {"value": round(units / sec / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{n} x one token through all {len(mats)} matvecs ({sec * 1e3:.2f} ms each, {n * sec:.1f} s)"}


def e2e_measure(args, lib, torch, dist, wl, w, copies, rows, rows_total, world, rank, device, stream, fm=None):
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
    if world == 1 or wl["shard"] == "replica":
        # the host entry point (x and y in host memory) on every rank's own block
        n_host = min(copies, 8)
        hosts = [w[i].cpu().numpy() for i in range(n_host)]
        for h in hosts:  # residency: first call uploads
            lib.matvec(t, rows, cols, h, x_host)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for k in range(args.steps):
            y_host = lib.matvec(t, rows, cols, hosts[k % n_host], x_host)
        sec = time.perf_counter() - t0
        if world > 1:
            tt = torch.tensor([sec], dtype=torch.float64, device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            sec = float(tt.item())
        sec /= args.steps
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
            if fm is not None:
                yf = fm.run(w[k % copies].data_ptr(), xd.data_ptr(), stream.cuda_stream)
            else:
                yf = sm.run(lambda xv, yl: lib.matvec_dev(t, rows, cols, w[k % copies].data_ptr(), xv.data_ptr(),
                                                          yl.data_ptr(), 1, stream.cuda_stream), xd, y, y_full)
            y_pin.copy_(yf, non_blocking=True)
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
            "d2h_bytes_per_step": 4 * rows_total,
            "path": "pinned H2D + " + ("nedo_gpu_matvec_allgather_dev + wait" if fm is not None else
                                       "nedo_gpu_matvec_dev + NCCL all-gather") + " + D2H",
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
        if wl.get("kind") == "sweep":
            run_sweep_arm(args, wl, world, rank, local_rank)
        else:
            run_gpu_arm(args, wl, world, rank, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
