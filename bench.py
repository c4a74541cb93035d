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
  decode_forward_24x1536
                       the device-resident decode forward pass of a NedoLM model
                       with the sweep's matrices (nedo_gpu_decoder_*: norms, fused
                       q|k|v and gate|up matvecs, RoPE, KV cache, attention, SiLU,
                       head + argmax in one CUDA graph per pass), greedy generation
                       with the loop on the device; GB/s of weights + KV cache per
                       pass and tokens/s.  The reference arm runs the reference's
                       own decode loop over the same GGUF.

Timing: W warm-up steps, then exactly K steps between a barrier +
cuda.synchronize on both sides, CUDA events on the launching stream, max over
ranks.  The K steps run as one CUDA graph (at N>1 with the all-gather of each
step inside it).  Weight copies rotate so the rotating set exceeds 4x L2 (each
step reads a weight that is not in L2).

At N=1 the line also carries `workloads`: every other configuration above
measured the same way in the same run (value, roofline fraction, clocks), and
at N>1 `sharded`: the row-sharded Q4_0 32768x32768 step with its time split
into the matvec and the gather wait.

`e2e` repeats the metric through the host entry point of the C ABI
(nedo_gpu_matvec: host x in, host y out, copies inside the timed region).
`cpu_baseline` times the reference's own CPU kernel (compiled from source into
oracle/_ref; the C restatement when that library is absent) on this host, and
as the checker of the same leg compares one output of each measured GPU
workload with the reference (`parity`).
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
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nedo.cpp_b200"))

import numpy as np  # noqa: E402

from nedo_gpu import blocks as B  # noqa: E402

METRIC = "Q8_0/Q4_0/F16 matvec HBM GB/s & % of B200 peak; prefill GEMM TFLOP/s @1-8 GPU"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1400.0
TOL = 1e-4  # |y_gpu - y_ref| <= TOL * sum_i |w_i x_i| per output

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
# the device-resident decode pass over the sweep's matrices: 12 heads x 128 with
# 12 KV heads (so q/k/v are 1536x1536 as in the sweep), the F16 64000x1536 head
# tied to the embedding, timed at positions 512.. of a running greedy decode
WORKLOADS["decode_forward_24x1536"] = dict(kind="decoder", type=B.Q8_0, layers=24, d=1536, heads=12, kv_heads=12,
                                           ff=4096, head=64000, context=4096, sliding=2048, pos=512, batch=1,
                                           shard="replica", argmax=True, rows=1536, cols=1536)
# measured beside the default line at N=1 (every configuration of the path)
SIDE_WORKLOADS = ["q8_0_4096x4096", "f16_head_128000x2048", "q4_0_32768x32768", "q8_0_prefill_512x4096x14336",
                  "decode_sweep_24x1536_b1", "decode_sweep_24x1536_b8", "decode_sweep_24x1536_b32",
                  "decode_forward_24x1536"]


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
    "q4_0_11008x4096": 25_470_208,
    "q8_0_4096x4096": 17_921_792,
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


def workload_config(name, wl, world):
    """The `config` of a line: identical in both arms (implementation details go to `setup`)."""
    if wl.get("kind") == "decoder":
        return {"workload": name,
                "description": f"NedoLM decode forward pass, {wl['layers']} layers, d_model {wl['d']}, "
                               f"{wl['heads']} heads x {wl['d'] // wl['heads']} ({wl['kv_heads']} KV heads), "
                               f"FFN {wl['ff']}, Q8_0 projections, F16 {wl['head']}x{wl['d']} head tied to the "
                               f"embedding, greedy, positions from {wl['pos']} (window {wl['sliding']})",
                "batch": 1, "weight_bytes_per_step": decoder_bytes(wl, wl["pos"])["weights"],
                "parallelism": "replicas" if world > 1 else "single"}
    if wl.get("kind") == "sweep":
        return {"workload": name,
                "description": f"{wl['layers']}-layer d_model {wl['d']} decoder step: "
                               f"{len(sweep_matrices(wl)) - 1} Q8_0 matvecs + F16 {wl['head']}x{wl['d']} head, "
                               f"{batch_of(wl)} token(s) per step",
                "batch": batch_of(wl), "weight_bytes_per_step": sum(r * B.row_bytes(t, c)
                                                                    for _, t, r, c in sweep_matrices(wl)),
                "parallelism": "replicas" if world > 1 else "single"}
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


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix="nedo_clocks_", suffix=".csv")
        os.close(fd)

    def start(self):
        try:
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
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline
# The reference processes a prompt as one matvec per token (src/model.cpp:262-266);
# a batch workload's CPU sample is this many of them per call.
CPU_BATCH_SAMPLE = 8


def checkers():
    """(reference or None, oracle) from oracle/ -- the CPU baseline leg's checkers."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    ref = None
    if O.Reference.available():
        ref = O.Reference()
        ref.set_threads(host_cores())
    return ref, O.Oracle()


def cpu_reference(type_, rows, cols, seed, nvec=1):
    """(callable, kind, cores) running the reference CPU kernel: `nvec` matvecs over one matrix."""
    ref, orc = checkers()
    w = B.gen_weight(type_, rows, cols, seed)
    xs = [B.gen_x(cols, seed + k) for k in range(nvec)]
    if ref is not None:
        return (lambda: [ref.matvec(type_, rows, cols, w, x) for x in xs]), "reference", host_cores()
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


def check_sample(sample):
    """Checker of the CPU baseline leg: one GPU output against the reference on
    the same bytes.  `sample` = list of (name, type, rows, cols, w bytes, x [k, cols],
    y_gpu [k, rows], argmax index or None)."""
    ref, orc = checkers()
    worst, checked, ok = 0.0, [], True
    argmax = None
    for name, t, rows, cols, w, x, y, idx in sample:
        for k in range(x.shape[0]):
            yr = (ref.matvec(t, rows, cols, w, x[k]) if ref is not None else orc.matvec(t, rows, cols, w, x[k]))
            absd = orc.abs_dot(t, rows, cols, w, x[k])
            err = np.abs(y[k].astype(np.float64) - yr.astype(np.float64))
            bound = TOL * absd
            r = float(np.max(err / np.maximum(bound, 1e-300)))
            worst = max(worst, r)
            ok = ok and bool(np.all(err <= bound))
            if idx is not None and k == 0:
                top = np.sort(yr.astype(np.float64))[-2:]
                ri = orc.argmax(yr)
                argmax = {"gpu": int(idx), "reference": int(ri), "equal": int(idx) == int(ri),
                          "top2_gap": float(top[1] - top[0]), "gap_over_bound": float((top[1] - top[0]) / max(
                              2 * TOL * float(absd.max()), 1e-300))}
                ok = ok and argmax["equal"]
        checked.append(f"{name} ({x.shape[0]} vector{'s' if x.shape[0] > 1 else ''})")
    out = {"ok": ok, "max_err_over_bound": round(worst, 5), "tolerance": f"{TOL} * sum|w*x| per output",
           "checker": "reference (oracle/_ref)" if ref is not None else "oracle (C restatement)",
           "checked": ", ".join(checked)}
    if argmax is not None:
        out["argmax"] = argmax
    return out


def run_reference_arm(args, wl, world, rank):
    if rank != 0:
        return
    if wl.get("kind") == "decoder":
        cb = decoder_cpu(wl, budget_s=min(20.0, 0.05 * args.steps + 2.0))
        line = {"metric": METRIC, "value": cb["value"], "unit": "GB/s", "impl": "reference", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic NedoLM GGUF (seeded weights)",
                "config": workload_config(args.workload, wl, world),
                "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                            "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if wl.get("kind") == "sweep":
        cb = sweep_cpu(wl, budget_s=min(20.0, 0.05 * args.steps + 2.0))
        line = {"metric": METRIC, "value": cb["value"], "unit": "GB/s", "impl": "reference", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF blocks)",
                "config": workload_config(args.workload, wl, world),
                "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                            "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    _, rows_total = shard_rows(wl, world)
    nvec = CPU_BATCH_SAMPLE if batch_of(wl) > 1 else 1
    fn, kind, cores = cpu_reference(wl["type"], rows_total, wl["cols"], seed=7, nvec=nvec)
    for _ in range(args.warmup):
        fn()
    # ~1 s soak (OpenMP thread pool and CPU clocks up), as the GPU arm soaks
    # before its timed region; it also sizes a step to ~25 ms of CPU work
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 1.0:
        fn()
        n += 1
    per_call = (time.perf_counter() - t0) / n
    reps = max(1, int(round(0.025 / per_call)))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(reps):
            fn()
    sec = (time.perf_counter() - t0) / (args.steps * reps)
    units, unit, scale = work_of(wl, rows_total, batch=nvec)
    value = units / sec / scale
    what = (f"{nvec} full {B.TYPE_NAMES[wl['type']]} {rows_total}x{wl['cols']} matvec"
            f"{'s (a sample of the batch, one per token)' if nvec > 1 else ''}")
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": unit, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3 * reps, 4),
        "higher_is_better": True, "scaling": "strong" if wl["shard"] == "strong" else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded GGUF blocks)",
        "config": workload_config(args.workload, wl, world),
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": cores, "kind": kind,
                         "sample": f"each step {reps} x {what} after a 1 s soak"},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ decoder
def decoder_bytes(wl, pos):
    """Algorithmic bytes of one decode pass at `pos`: every weight once (the
    embedding: one row), the KV cache rows attention reads and the new ones."""
    d, ff, L = wl["d"], wl["ff"], wl["layers"]
    hd = d // wl["heads"]
    qd, kvd = wl["heads"] * hd, wl["kv_heads"] * hd
    rb = B.row_bytes
    t = wl["type"]
    layer = (qd + 2 * kvd) * rb(t, d) + d * rb(t, qd) + 2 * ff * rb(t, d) + d * rb(t, ff) + 2 * 4 * d
    weights = L * layer + wl["head"] * 2 * d + 4 * d + 2 * d
    window = min(wl["sliding"] or wl["context"], wl["context"])
    nctx = min(pos + 1, window)
    kv = L * (nctx + 1) * kvd * 4 * 2
    return {"weights": weights, "kv": kv, "total": weights + kv}


_DECODER_FILE = {}


def decoder_model(wl):
    """Path of the synthetic GGUF of the decoder workload (built once per process)."""
    key = id(wl)
    if key not in _DECODER_FILE:
        from nedo_gpu import gguf as G

        path = os.path.join(tempfile.mkdtemp(prefix="nedo_bench_"), "decoder.gguf")
        G.synthetic_model(path, dim=wl["d"], layers=wl["layers"], heads=wl["heads"], kv_heads=wl["kv_heads"],
                          ffn=wl["ff"], vocab=wl["head"], context=wl["context"], sliding=wl["sliding"],
                          wtype=wl["type"], emb_type=B.F16, tied=True, norm_type=0, shared_layers=True, seed=5)
        _DECODER_FILE[key] = path
    return _DECODER_FILE[key]


REF_DECODE = os.path.join(ROOT, "oracle", "_ref", "ref_decode")


def ref_decode_run(path, prompt, max_new, logits=True):
    """(seconds, logits [passes, vocab] or None, ids) of the reference's own decode
    loop (oracle/_ref/ref_decode: src/model.cpp generate_ids, greedy)."""
    out = os.path.join(tempfile.mkdtemp(prefix="nedo_ref_"), "out.bin")
    env = dict(os.environ, OMP_NUM_THREADS=str(host_cores()))
    t0 = time.perf_counter()
    subprocess.run([REF_DECODE, path, out, str(max_new), "0", "0", "0", "0"] + [str(t) for t in prompt],
                   check=True, env=env, stdout=subprocess.DEVNULL)
    sec = time.perf_counter() - t0
    b = open(out, "rb").read()
    a = np.frombuffer(b, dtype=np.uint32)
    steps, vocab = int(a[0]), int(a[1])
    lg = np.frombuffer(b, dtype=np.float32, count=steps * vocab, offset=8).reshape(steps, vocab) if logits else None
    n = int(a[2 + steps * vocab])
    return sec, lg, [int(v) for v in a[3 + steps * vocab:3 + steps * vocab + n]]


def decoder_cpu(wl, budget_s=10.0):
    """The reference's decode loop on this host: seconds per pass from two runs
    (one pass, then 1 + m passes) so the model load cancels."""
    if not os.path.exists(REF_DECODE):
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref/ref_decode not built (make -C oracle ref)"}
    path = decoder_model(wl)
    t1, _, _ = ref_decode_run(path, [5], 0, logits=False)
    m = 8
    tm, _, _ = ref_decode_run(path, [5], m, logits=False)
    per = max((tm - t1) / m, 1e-6)
    m = int(min(max(8, budget_s / per), 256))
    tm, _, ids = ref_decode_run(path, [5], m, logits=False)
    t1, _, _ = ref_decode_run(path, [5], 0, logits=False)
    passes = len(ids)  # passes after the first: one per generated id (eos may stop it early)
    per = max((tm - t1) / max(passes, 1), 1e-6)
    byts = decoder_bytes(wl, passes // 2)["total"]
    return {"value": round(byts / per / 1e9, 3), "unit": "GB/s", "cores": host_cores(), "kind": "reference",
            "tokens_per_s": round(1.0 / per, 2),
            "sample": f"the reference's generate_ids (oracle/_ref/ref_decode) over the same GGUF: {passes} greedy "
                      f"passes at positions 1..{passes} ({per * 1e3:.2f} ms each), the one-pass run subtracted"}


def measure_decoder(ctx, name, steps, keep_sample=False):
    """The device-resident decode pass: greedy generation with the loop on the
    device, `steps` passes at positions wl['pos'].. after filling the KV cache."""
    torch, lib = ctx.torch, ctx.lib
    from nedo_gpu import gguf as G
    from nedo_gpu.decoder import Decoder

    wl = WORKLOADS[name]
    g = G.GgufFile(decoder_model(wl))
    dec = Decoder.from_gguf(g, lib)
    dec.set_stream(ctx.stream.cuda_stream)
    p0 = wl["pos"]
    steps = max(1, min(steps, wl["context"] - p0 - 1, 200))
    ids = dec.generate(5, 0, p0)  # positions 0 .. p0-1: the cache the timed passes attend over
    tok = ids[-1]
    sampler = ClockSampler(ctx.local_rank)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    while time.perf_counter() < soak_end:
        dec.generate(tok, p0, steps)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed")
    ev0.record(ctx.stream)
    gen = dec.generate(tok, p0, steps)
    ev1.record(ctx.stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    ctx.barrier()
    ms = ctx.max_over_ranks(ev0.elapsed_time(ev1)) / steps
    clocks = sampler.stop()
    byts = decoder_bytes(wl, p0 + steps // 2)
    value = byts["total"] / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    # e2e: the same passes as host calls (token in, greedy id out, one round trip each)
    t0 = time.perf_counter()
    t = tok
    for k in range(steps):
        t, _ = dec.forward(t, p0 + k, logits=False)
    e2e_sec = ctx.max_over_ranks(time.perf_counter() - t0) / steps
    mats = 4 * wl["layers"] + 1
    out = {"value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 6), "steps": steps,
           "tokens_per_s": round(1e3 / ms, 2), "launches_per_step": 3 + 5 * wl["layers"] + 1,
           "matvecs_per_step": mats,
           "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(value / peak, 4), "traffic": None, "peak_source": peak_kind,
                        "launch_us": round(ms * 1e3, 3), "bytes_per_step": byts},
           "clocks": clocks,
           "e2e": {"value": round(byts["total"] / e2e_sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 16,
                   "d2h_bytes_per_step": 12 + 16, "ms_per_step": round(e2e_sec * 1e3, 4),
                   "tokens_per_s": round(1.0 / e2e_sec, 2),
                   "path": "nedo_gpu_decoder_forward per token (token id in, greedy id out)"},
           "generated": gen[:8]}
    if keep_sample:
        out["parity"] = decoder_parity(dec, wl)
    dec.close()
    g.close()
    return out


def decoder_parity(dec, wl, prompt=(5, 300, 301, 302), tol=2e-4):
    """Checker of the CPU baseline leg: the decoder's logits on a short sequence
    against the reference's own decode loop on the same GGUF."""
    if not os.path.exists(REF_DECODE):
        return {"ok": None, "checker": "unavailable: oracle/_ref/ref_decode not built"}
    _, ref, _ = ref_decode_run(decoder_model(wl), list(prompt), 0)
    dec.reset()
    worst, same = 0.0, True
    for pos, t in enumerate(prompt):
        pick, lg = dec.forward(t, pos)
        worst = max(worst, float(np.abs(lg - ref[pos]).max() / np.abs(ref[pos]).max()))
        same = same and pick == int(np.argmax(ref[pos]))
    return {"ok": bool(worst <= tol and same), "max_logit_err_over_max_logit": worst, "tolerance": tol,
            "argmax_equal": same, "checker": "reference decode loop (oracle/_ref/ref_decode)",
            "checked": f"{len(prompt)} passes, logits of each"}


# ------------------------------------------------------------------ GPU arm
class Ctx:
    """Per-process GPU state shared by the measurements."""

    def __init__(self, args, world, rank, local_rank):
        import torch
        import torch.distributed as dist

        import nedo_gpu

        self.torch, self.dist = torch, dist
        self.args, self.world, self.rank, self.local_rank = args, world, rank, local_rank
        torch.cuda.set_device(local_rank)
        self.device = torch.device("cuda", local_rank)
        self.lib = nedo_gpu.load()
        # Programmatic dependent launch: each matvec starts streaming its weight
        # while the previous launch drains (x is read only after it completed).
        self.lib.set_pdl(True)
        self.stream = torch.cuda.Stream(device=self.device)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        tt = self.torch.tensor([v], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(tt, op=self.dist.ReduceOp.MAX)
        return float(tt.item())

    def timed_graph(self, graph, clocks=True):
        """(ms of one replay, clocks): 1 s soak, then one replay between barriers + syncs."""
        torch = self.torch
        sampler = ClockSampler(self.local_rank) if clocks else None
        if sampler:
            sampler.start()
        soak_end = time.perf_counter() + 1.0
        while time.perf_counter() < soak_end:  # clocks under load before the timed region
            graph.replay()
            torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        torch.cuda.synchronize()
        # the NVTX range marks the timed launches for profilers (ncu --nvtx --nvtx-include timed/)
        torch.cuda.nvtx.range_push("timed")
        with torch.cuda.stream(self.stream):
            ev0.record(self.stream)
            graph.replay()
            ev1.record(self.stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        self.barrier()
        ms = self.max_over_ranks(ev0.elapsed_time(ev1))
        return ms, (sampler.stop() if sampler else None)


def launches_per_call(plan, nb):
    """Kernels of this library one matvec_dev call launches (the library's own count)."""
    return plan["launches"]


def measure_matvec(ctx, name, steps, keep_sample=False):
    """One matvec workload on this GPU alone (N=1 replica semantics): the value,
    the roofline, clocks and (optionally) a sample for the checker."""
    torch, lib = ctx.torch, ctx.lib
    wl = WORKLOADS[name]
    t, rows, cols = wl["type"], wl["rows"], wl["cols"]
    nb = batch_of(wl)
    rb = B.row_bytes(t, cols)
    copies = max(1, math.ceil(4 * L2_BYTES / (rows * rb)))
    w = B.gen_weight_torch(torch, t, rows, cols, copies, seed=1000 + ctx.rank, device=ctx.device)
    gx = torch.Generator(device=ctx.device)
    gx.manual_seed(7)
    x = torch.randn((nb, cols) if nb > 1 else cols, generator=gx, device=ctx.device, dtype=torch.float32)
    y = torch.empty((nb, rows) if nb > 1 else rows, dtype=torch.float32, device=ctx.device)
    idx = torch.zeros(1, dtype=torch.int64, device=ctx.device)
    val = torch.zeros(1, dtype=torch.float32, device=ctx.device)
    plan = lib.plan_info(t, rows, cols, nb)
    lib.reserve(t, rows, cols, nb)

    def launch(k, s):
        wp = w[k % copies].data_ptr()
        if wl["argmax"]:
            lib.matvec_argmax_dev(t, rows, cols, wp, x.data_ptr(), y.data_ptr(), idx.data_ptr(), val.data_ptr(), s)
        else:
            lib.matvec_dev(t, rows, cols, wp, x.data_ptr(), y.data_ptr(), nb, s)

    with torch.cuda.stream(ctx.stream):
        for k in range(max(3, ctx.args.warmup)):
            launch(k, ctx.stream.cuda_stream)
    torch.cuda.synchronize()
    lib.status(ctx.stream.cuda_stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=ctx.stream):
        for k in range(steps):
            launch(k, torch.cuda.current_stream().cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    ms, clocks = ctx.timed_graph(graph)
    lib.status(ctx.stream.cuda_stream)
    del graph
    ms_per_step = ms / steps
    units, unit, scale = work_of(wl, rows)
    value = units / (ms_per_step * 1e-3) / scale
    tensor = nb > 1
    peak, peak_kind = peaks(tensor)
    out = {"value": round(value, 2), "unit": unit, "ms_per_step": round(ms_per_step, 6), "plan": plan,
           "roofline": {"bound": "tensor" if tensor else "hbm", "achieved": round(value, 1), "peak": peak,
                        "unit": unit, "frac": round(value / peak, 4), "traffic": NCU_TRAFFIC_BYTES.get(name),
                        "peak_source": peak_kind, "launch_us": round(ms_per_step * 1e3, 3),
                        ("flops_per_step" if tensor else "bytes_per_launch"): units},
           "clocks": clocks, "copies": copies}
    if keep_sample:
        # one eager launch on copy 0 for the checker (a sample of 8 tokens of a batch)
        with torch.cuda.stream(ctx.stream):
            launch(0, ctx.stream.cuda_stream)
        torch.cuda.synchronize()
        kk = min(nb, CPU_BATCH_SAMPLE)
        xs = x.reshape(nb, cols)[:kk].cpu().numpy()
        ys = y.reshape(nb, rows)[:kk].cpu().numpy()
        out["sample"] = [(name, t, rows, cols, w[0].cpu().numpy(), xs, ys,
                          int(idx.item()) if wl["argmax"] else None)]
    out["_state"] = (w, copies, x, y, launch, plan)
    return out


def measure_sweep(ctx, name, steps_req, keep_sample=False):
    """Decode sweep: every matvec of one decoder step (plus the head) per step,
    all weights resident (918 MB: more than 4x L2, so each step reads HBM)."""
    torch, lib = ctx.torch, ctx.lib
    wl = WORKLOADS[name]
    nb = batch_of(wl)
    mats = sweep_matrices(wl)
    ws = [B.gen_weight_torch(torch, t, r, c, 1, seed=2000 + 7 * i + ctx.rank, device=ctx.device)[0]
          for i, (_, t, r, c) in enumerate(mats)]
    d, ff = wl["d"], wl["ff"]
    g = torch.Generator(device=ctx.device)
    g.manual_seed(7)
    xd = torch.randn((nb, d), generator=g, device=ctx.device)
    xf = torch.randn((nb, ff), generator=g, device=ctx.device)
    yd = torch.empty((nb, d), device=ctx.device)
    yf = torch.empty((nb, ff), device=ctx.device)
    logits = torch.empty((nb, wl["head"]), device=ctx.device)
    idx = torch.zeros(1, dtype=torch.int64, device=ctx.device)
    val = torch.zeros(1, dtype=torch.float32, device=ctx.device)
    for _, t, r, c in mats:
        lib.reserve(t, r, c, nb)

    def one(i, s):
        nm, t, r, c = mats[i]
        x = xf if c == ff else xd
        y = logits if nm == "head" else (yf if r == ff else yd)
        if nm == "head" and wl["argmax"]:
            lib.matvec_argmax_dev(t, r, c, ws[i].data_ptr(), x.data_ptr(), y.data_ptr(), idx.data_ptr(),
                                  val.data_ptr(), s)
        else:
            lib.matvec_dev(t, r, c, ws[i].data_ptr(), x.data_ptr(), y.data_ptr(), nb, s)

    def step(s):
        for i in range(len(mats)):
            one(i, s)

    with torch.cuda.stream(ctx.stream):
        for _ in range(max(3, ctx.args.warmup)):
            step(ctx.stream.cuda_stream)
    torch.cuda.synchronize()
    lib.status(ctx.stream.cuda_stream)
    steps = max(1, min(steps_req, 50))  # about 1 ms per step
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=ctx.stream):
        for _ in range(steps):
            step(torch.cuda.current_stream().cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    ms, clocks = ctx.timed_graph(graph)
    ms_per_step = ms / steps
    del graph
    lib.status(ctx.stream.cuda_stream)

    # per matrix kind: the 24 layers' launches of one kind (or the head) as one graph
    kinds = {}
    for i, (nm, t, r, c) in enumerate(mats):
        kinds.setdefault(nm.rstrip("0123456789"), []).append(i)
    per_kind = {}
    for kind, ids in kinds.items():
        kg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kg, stream=ctx.stream):
            for _ in range(3):
                for i in ids:
                    one(i, torch.cuda.current_stream().cuda_stream)
        kg.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(ctx.stream):
            a.record(ctx.stream)
            kg.replay()
            b.record(ctx.stream)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / (3 * len(ids))
        _, t, r, c = mats[ids[0]]
        byts = r * B.row_bytes(t, c) + nb * 4 * (r + c)
        per_kind[f"{kind} {B.TYPE_NAMES[t]} {r}x{c}"] = {"us": round(us, 3), "GB/s": round(byts / us / 1e3, 1),
                                                       "path": lib.plan_info(t, r, c, nb)["path"]}
        del kg

    units = sweep_bytes(wl, nb)
    value = units / (ms_per_step * 1e-3) / 1e9
    peak, peak_kind = peaks()
    launches = sum(launches_per_call(lib.plan_info(t, r, c, nb), nb) for _, t, r, c in mats)
    out = {"value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms_per_step, 6), "steps": steps,
           "per_matrix": per_kind, "launches_per_step": launches,
           "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(value / peak, 4), "traffic": None, "peak_source": peak_kind,
                        "launch_us": round(ms_per_step * 1e3, 3), "bytes_per_step": units},
           "clocks": clocks}
    if keep_sample:
        with torch.cuda.stream(ctx.stream):
            step(ctx.stream.cuda_stream)
        torch.cuda.synchronize()
        kk = min(nb, CPU_BATCH_SAMPLE)
        sample = []
        # one matrix of each kind, recomputed eagerly into its own output
        for kind in ("q", "gate", "down", "head"):
            i = kinds[kind][0]
            nm, t, r, c = mats[i]
            x = xf if c == ff else xd
            yo = torch.empty((nb, r), device=ctx.device)
            if nm == "head" and wl["argmax"]:
                lib.matvec_argmax_dev(t, r, c, ws[i].data_ptr(), x.data_ptr(), yo.data_ptr(), idx.data_ptr(),
                                      val.data_ptr(), ctx.stream.cuda_stream)
            else:
                lib.matvec_dev(t, r, c, ws[i].data_ptr(), x.data_ptr(), yo.data_ptr(), nb, ctx.stream.cuda_stream)
            torch.cuda.synchronize()
            sample.append((f"{nm} {B.TYPE_NAMES[t]} {r}x{c}", t, r, c, ws[i].cpu().numpy(), x[:kk].cpu().numpy(),
                           yo[:kk].cpu().numpy(), int(idx.item()) if (nm == "head" and wl["argmax"]) else None))
        out["sample"] = sample
    out["_state"] = (mats, ws, xd, logits, step)
    return out


def side_record(r):
    keep = ("value", "unit", "ms_per_step", "roofline", "clocks", "parity", "per_matrix", "launches_per_step",
            "tokens_per_s", "e2e")
    return {k: r[k] for k in keep if k in r}


def e2e_matvec(ctx, wl, w, copies, rows, rows_total, fm=None):
    torch, lib, dist = ctx.torch, ctx.lib, ctx.dist
    world = ctx.world
    stream = ctx.stream
    t, cols = wl["type"], wl["cols"]
    nb = batch_of(wl)
    steps = ctx.args.steps
    if nb > 1:
        # a prompt-sized batch end to end through the host entry point
        # (nedo_gpu_matvec_batch: host x in, host y out, resident weight)
        x_host = np.random.default_rng(7).standard_normal((nb, cols), dtype=np.float32)
        n_host = min(copies, 4)
        hosts = [w[i].cpu().numpy() for i in range(n_host)]
        for h in hosts:
            lib.matvec_batch(t, rows, cols, h, x_host)
        ctx.barrier()
        t0 = time.perf_counter()
        reps = max(1, min(steps, 50))
        for k in range(reps):
            y_host = lib.matvec_batch(t, rows, cols, hosts[k % n_host], x_host)
        sec = ctx.max_over_ranks(time.perf_counter() - t0) / reps
        assert y_host.shape == (nb, rows)
        for h in hosts:
            lib.weight_evict(h)
        units, unit, scale = work_of(wl, rows_total)
        return {"value": round(units / sec / scale, 2), "unit": unit, "h2d_bytes_per_step": 4 * nb * cols,
                "d2h_bytes_per_step": 4 * nb * rows, "path": "nedo_gpu_matvec_batch (host pointers, resident weight)",
                "ms_per_step": round(sec * 1e3, 4)}
    x_host = np.random.default_rng(7).standard_normal(cols, dtype=np.float32)
    if world == 1 or wl["shard"] == "replica":
        # the host entry point (x and y in host memory) on every rank's own block
        n_host = min(copies, 8)
        hosts = [w[i].cpu().numpy() for i in range(n_host)]
        for h in hosts:  # residency: first call uploads
            lib.matvec(t, rows, cols, h, x_host)
        ctx.barrier()
        t0 = time.perf_counter()
        for k in range(steps):
            y_host = lib.matvec(t, rows, cols, hosts[k % n_host], x_host)
        sec = ctx.max_over_ranks(time.perf_counter() - t0) / steps
        assert y_host.shape == (rows,)
        for h in hosts:
            lib.weight_evict(h)
        bytes_total = algorithmic_bytes(t, rows_total, cols)
        return {"value": round(bytes_total / sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * cols,
                "d2h_bytes_per_step": 4 * rows, "path": "nedo_gpu_matvec (host pointers, resident weight)",
                "ms_per_step": round(sec * 1e3, 4)}
    # N > 1: pinned host x -> device, shard matvec, all-gather, full y -> host
    x_pin = torch.from_numpy(x_host).pin_memory()
    y_pin = torch.empty(rows_total, dtype=torch.float32).pin_memory()
    xd = torch.empty(cols, dtype=torch.float32, device=ctx.device)
    y = torch.empty(rows, dtype=torch.float32, device=ctx.device)
    y_full = torch.empty(rows_total, dtype=torch.float32, device=ctx.device)

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
    for k in range(steps):
        one(k)
    sec = ctx.max_over_ranks(time.perf_counter() - t0) / steps
    bytes_total = algorithmic_bytes(t, rows_total, cols)
    return {"value": round(bytes_total / sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * cols,
            "d2h_bytes_per_step": 4 * rows_total,
            "path": "pinned H2D + " + ("nedo_gpu_matvec_allgather_dev + wait" if fm is not None else
                                       "nedo_gpu_matvec_dev + NCCL all-gather") + " + D2H",
            "ms_per_step": round(sec * 1e3, 4)}


def e2e_sweep(ctx, wl, state):
    torch = ctx.torch
    mats, ws, xd, logits, step = state
    nb = batch_of(wl)
    d = wl["d"]
    x_pin = torch.randn((nb, d)).pin_memory()
    l_pin = torch.empty((nb, wl["head"])).pin_memory()
    reps = 5

    def once():
        with torch.cuda.stream(ctx.stream):
            xd.copy_(x_pin, non_blocking=True)
            step(ctx.stream.cuda_stream)
            l_pin.copy_(logits, non_blocking=True)
        ctx.stream.synchronize()

    once()
    t0 = time.perf_counter()
    for _ in range(reps):
        once()
    sec = ctx.max_over_ranks(time.perf_counter() - t0) / reps
    units = sweep_bytes(wl, nb) * ctx.world
    return {"value": round(units / sec / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * nb * d,
            "d2h_bytes_per_step": 4 * nb * wl["head"], "path": "pinned H2D + 169 nedo_gpu_matvec_dev + D2H",
            "ms_per_step": round(sec * 1e3, 4)}


def measure_sharded(ctx, name, steps):
    """The row-sharded matvec at N = world ranks (strong scaling): matvec + the
    fused all-gather (NCCL where that kernel does not take the shape).  Returns
    the whole-job value and the per-step time split into the matvec alone and
    the gather (the step minus the matvec, max over ranks)."""
    torch, lib = ctx.torch, ctx.lib
    from nedo_gpu.shard import FusedShardedMatvec, ShardedMatvec

    wl = WORKLOADS[name]
    t, cols = wl["type"], wl["cols"]
    rows, rows_total = shard_rows(wl, ctx.world)
    rb = B.row_bytes(t, cols)
    copies = max(1, math.ceil(4 * L2_BYTES / (rows * rb)))
    w = B.gen_weight_torch(torch, t, rows, cols, copies, seed=1000 + ctx.rank, device=ctx.device)
    gx = torch.Generator(device=ctx.device)
    gx.manual_seed(7)
    x = torch.randn(cols, generator=gx, device=ctx.device, dtype=torch.float32)
    y = torch.empty(rows, dtype=torch.float32, device=ctx.device)
    y_full = torch.empty(rows_total, dtype=torch.float32, device=ctx.device)
    plan = lib.plan_info(t, rows, cols, 1)
    fm = sm = None
    if plan.get("path") == 4:
        fm = FusedShardedMatvec(lib, t, rows_total, cols, ctx.device)
        collective = "fused: rows stored on every peer over NVLink by the matvec kernel + completion wait"
    else:
        sm = ShardedMatvec(t, rows_total, cols)
        collective = "NCCL all-gather of the y slices"

    def local(k, s):
        lib.matvec_dev(t, rows, cols, w[k % copies].data_ptr(), x.data_ptr(), y.data_ptr(), 1, s)

    def step(k):
        if fm is not None:
            fm.run(w[k % copies].data_ptr(), x.data_ptr(), torch.cuda.current_stream().cuda_stream)
        else:
            sm.run(lambda xv, yl: local(k, torch.cuda.current_stream().cuda_stream), x, y, y_full)

    with torch.cuda.stream(ctx.stream):
        for k in range(4):
            step(k)
    torch.cuda.synchronize()
    lib.status(ctx.stream.cuda_stream)
    n = steps + (steps & 1)  # even: the fused path alternates two gathered buffers
    g_local = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_local, stream=ctx.stream):
        for k in range(n):
            local(k, torch.cuda.current_stream().cuda_stream)
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step, stream=ctx.stream):
        for k in range(n):
            step(k)
    g_local.replay()
    g_step.replay()
    torch.cuda.synchronize()
    ctx.barrier()
    ms_step, clocks = ctx.timed_graph(g_step)
    ms_local, _ = ctx.timed_graph(g_local, clocks=False)
    lib.status(ctx.stream.cuda_stream)
    del g_step, g_local  # the step graph may hold NCCL calls: released before the process group
    per = ms_step / n
    units = algorithmic_bytes(t, rows_total, cols)
    value = units / (per * 1e-3) / 1e9
    return {"workload": name, "value": round(value, 2), "unit": "GB/s", "scaling": "strong",
            "ms_per_step": round(per, 6), "matvec_ms": round(ms_local / n, 6),
            "gather_ms": round(max(per - ms_local / n, 0.0), 6), "collective": collective,
            "rows_per_gpu": rows, "n_gpus": ctx.world, "clocks": clocks,
            "_state": (w, copies, fm)}


def run_gpu_arm(args, wl, world, rank, local_rank):
    ctx = Ctx(args, world, rank, local_rank)
    torch = ctx.torch
    name = args.workload
    check = rank == 0 and world == 1 and not args.no_cpu_baseline
    setup = {}
    if wl.get("kind") == "decoder":
        r = measure_decoder(ctx, name, args.steps, keep_sample=check)
        line = {"metric": METRIC, "value": round(r["value"] * world, 2), "unit": "GB/s", "n_gpus": world,
                "steps": r["steps"], "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
                "data": "synthetic NedoLM GGUF (seeded weights, layers sharing one set of bytes)",
                "config": workload_config(name, wl, world),
                "setup": {"l2": "918 MB of weights resident: each pass streams them from HBM (> 4x L2)",
                          "graph": "one CUDA graph per pass (3 + 5 x layers launches: norms and SiLU fused into the projections; + the on-device advance)",
                          "pdl": True, "tokens_per_s": r["tokens_per_s"]},
                "roofline": r["roofline"], "e2e": r["e2e"], "gpu_launches": r["steps"] * r["launches_per_step"],
                "clocks": r["clocks"]}
        if check:
            line["cpu_baseline"] = decoder_cpu(wl)
            line["parity"] = r["parity"]
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    if wl.get("kind") == "sweep":
        r = measure_sweep(ctx, name, args.steps, keep_sample=check)
        e2e = e2e_sweep(ctx, wl, r["_state"])
        value_total = r["value"] * world
        line = {"metric": METRIC, "value": round(value_total, 2), "unit": "GB/s", "n_gpus": world,
                "steps": r["steps"], "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
                "data": "synthetic (seeded GGUF blocks, torch.Generator on device)",
                "config": workload_config(name, wl, world),
                "setup": {"l2": "918 MB of weights, all resident: each step streams them from HBM (> 4x L2)",
                          "graph": f"{r['steps']} steps of {len(sweep_matrices(wl))} matvecs captured as one CUDA graph",
                          "pdl": True, "per_matrix": r["per_matrix"]},
                "roofline": r["roofline"], "e2e": e2e, "gpu_launches": r["steps"] * r["launches_per_step"],
                "clocks": r["clocks"]}
        if check:
            line["cpu_baseline"] = sweep_cpu(wl, budget_s=10.0)
            line["parity"] = check_sample(r["sample"])
        if rank == 0:
            print(json.dumps(line), flush=True)
        return

    t, cols = wl["type"], wl["cols"]
    rows, rows_total = shard_rows(wl, world)
    nb = batch_of(wl)
    if world == 1 or wl["shard"] == "replica":
        r = measure_matvec(ctx, name, args.steps, keep_sample=check)
        w, copies, x, y, launch, plan = r["_state"]
        value_total = r["value"] * world if world > 1 else r["value"]
        ms_per_step = r["ms_per_step"]
        clocks = r["clocks"]
        roofline = r["roofline"]
        fm = None
        collective = None
        if world > 1:
            # replicas: the max-over-ranks time of every rank's own block
            value_total = work_of(wl, rows_total)[0] / (ms_per_step * 1e-3) / work_of(wl, rows_total)[2]
    else:
        r = measure_sharded(ctx, name, args.steps)
        w, copies, fm = r["_state"]
        plan = ctx.lib.plan_info(t, rows, cols, 1)
        value_total = r["value"]
        ms_per_step = r["ms_per_step"]
        clocks = r["clocks"]
        per_launch, unit, scale = work_of(wl, rows)
        achieved = per_launch / (r["matvec_ms"] * 1e-3) / scale
        peak, peak_kind = peaks()
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": unit,
                    "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_kind,
                    "launch_us": round(r["matvec_ms"] * 1e3, 3), "bytes_per_launch": per_launch}
        collective = r["collective"]
        setup["gather_ms"] = r["gather_ms"]
        setup["matvec_ms"] = r["matvec_ms"]
    setup.update({"l2": f"{copies} rotating weight copies ({copies * rows * B.row_bytes(t, cols) / 2**20:.0f} MiB "
                        f"per GPU, > 4x L2)",
                  "graph": "K steps (matvec" + (" + all-gather" if collective else "") +
                           ") captured as one CUDA graph",
                  "pdl": True, "plan": plan})
    if collective:
        setup["collective"] = collective
    e2e = e2e_matvec(ctx, wl, w, copies, rows, rows_total, fm)
    path = plan.get("path")
    line = {
        "metric": METRIC, "value": round(value_total, 2), "unit": roofline["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if wl["shard"] == "strong" else "weak", "vs_baseline": None,
        # block dots on the int8 tensor pipe (exact int32) for the int8 plan; fp16
        # operands with fp32 accumulation on tcgen05 for batches; fp32 FMA otherwise
        "dtype": {4: "int8", 5: "f16"}.get(path, "f32"),
        "data": "synthetic (seeded GGUF blocks, torch.Generator on device)",
        "config": workload_config(name, wl, world), "setup": setup,
        "roofline": roofline, "e2e": e2e,
        # one matvec kernel per step (argmax fused into it); batches: x -> fp16, the GEMM (+ split-K fold)
        "gpu_launches": args.steps * launches_per_call(plan, nb),
        "clocks": clocks,
    }
    if check:
        line["cpu_baseline"] = cpu_baseline(wl, rows_total)
        line["parity"] = check_sample(r["sample"])
    del r
    if world == 1 and not args.no_side:
        # every other configuration of the path, measured the same way in this run
        side = {}
        for other in SIDE_WORKLOADS:
            if other == name:
                continue
            torch.cuda.empty_cache()
            ow = WORKLOADS[other]
            if ow.get("kind") == "decoder":
                rr = measure_decoder(ctx, other, 50, keep_sample=check)
            elif ow.get("kind") == "sweep":
                rr = measure_sweep(ctx, other, 20, keep_sample=check)
            else:
                rr = measure_matvec(ctx, other, 20 if batch_of(ow) == 1 else 10, keep_sample=check)
            if check and "sample" in rr:
                rr["parity"] = check_sample(rr.pop("sample"))
            side[other] = side_record(rr)
            del rr
        line["workloads"] = side
    elif world > 1 and name != "q4_0_32768x32768" and not args.no_side:
        # the collective of the path: row-sharded Q4_0 32768x32768 at this N
        torch.cuda.empty_cache()
        rs = measure_sharded(ctx, "q4_0_32768x32768", 20)
        rs.pop("_state")
        line["sharded"] = rs
    if rank == 0:
        print(json.dumps(line), flush=True)


def sweep_cpu(wl, budget_s=10.0):
    """The reference CPU kernels over one token of the sweep (all 169 matvecs)."""
    ref, orc = checkers()
    mats = sweep_matrices(wl)
    data = [(t, r, c, B.gen_weight(t, r, c, 3000 + i), B.gen_x(c, 3000 + i)) for i, (_, t, r, c) in enumerate(mats)]
    if ref is not None:
        kind, cores = "reference", host_cores()
    else:
        ref, kind, cores = orc, "port", 1

    def fn():
        for t, r, c, w, x in data:
            ref.matvec(t, r, c, w, x)

    sec, n = time_cpu(fn, budget_s, 1000)
    units = sweep_bytes(wl, 1)
    return {"value": round(units / sec / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{n} x one token through all {len(mats)} matvecs ({sec * 1e3:.2f} ms each, {n * sec:.1f} s)"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="q4_0_11008x4096", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg (and its checker)")
    ap.add_argument("--no-side", action="store_true", help="measure only --workload (no `workloads` / `sharded`)")
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
