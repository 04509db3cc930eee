#!/usr/bin/env python3
"""Benchmark of the vlak hot path on B200 (one JSON line on rank 0).

Workload: one flow-matching chunk of SmolVLA
action-expert self-attention -- 16 expert layers x 10 denoising steps = 160
calls of vlak::fused_attention_gqa_v4 on q (B, 50, 15, 64), k/v (B, 291, 5, 64)
bf16 with the analytic prefix/staircase mask (P = 241) -- over B = 2048 policy
queries, batch-sharded over the N GPUs of one node (strong scaling: total work
fixed), followed by one NCCL all-gather of the chunk's output. A step is one
chunk; the 160 calls of a step are replayed from a CUDA graph, as the compiled
model runs them.

Metric: whole-job attention calls per second (one call = one B=2048 call,
all shards); µs/call = 1e6 / value. Inputs: 16 per-layer input sets (one per
expert layer), each larger than L2 at every N, rotated through the chunk, so
every call reads cold K/V/Q from HBM.

Extra keys: roofline of the attention kernel (HBM-bound at this shape) and its
tensor-pipe fraction, e2e through the torch op with pinned host buffers, the
CPU baseline (oracle port on host cores, rank 0, N=1), clocks sampled during the
timed region, and a softmax line (config C2 wide rows, 1 GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "vla-kernels_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from kernels import workloads as wl  # noqa: E402
from kernels.batch_shard import shard  # noqa: E402

GLOBAL_B = 2048
LAYERS, FLOW_STEPS = 16, 10
CALLS_PER_STEP = LAYERS * FLOW_STEPS
METRIC = "GQA attn calls/s (SmolVLA expert self-attn C5, B=2048, 160 calls/chunk; us/call = 1e6/value)"
UNIT = "calls/s"
C5_WORKLOAD = ("C5: expert self-attn q(B,50,15,64) k/v(B,291,5,64) P=241, B=2048 "
               "(sharded over the GPUs, then one NCCL all-gather)")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------- helpers

def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


# The committed ncu capture of the attention kernel: the raw-page metrics of
# two launches on the C3/C5 shapes at this batch (larger than L2), read by
# roofline.py. DRAM traffic grows with the number of batch elements, so it is
# scaled to a launch's batch.
NCU_ATTN_CSV = os.path.join(REPO, "profiles", "gqa_attention_sm100_c5_b512.csv")
NCU_ATTN_BATCH = 512


def attention_traffic(batch: int):
    """DRAM bytes (read + write) per launch of the attention kernel at
    `batch`, from the committed ncu capture, or None."""
    import roofline

    if not os.path.exists(NCU_ATTN_CSV):
        return None
    t = roofline.kernel_traffic(NCU_ATTN_CSV, "gqa_attention_sm100")
    return None if t is None else int(round(t * batch / NCU_ATTN_BATCH))


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------- our arm

def bench_ours(args, rank, world, local):
    from kernels.attention import fused_attention_gqa_v4

    lo, hi = shard(GLOBAL_B, rank, world)
    B = hi - lo
    shape = wl.expert_shape(B)
    scale = 0.125
    # 16 per-layer input sets (seeded by layer and shard offset)
    sets = [wl.attn_inputs(shape, seed=1000 * layer + lo) for layer in range(LAYERS)]

    def chunk():
        out = None
        for step in range(FLOW_STEPS):
            for layer in range(LAYERS):
                q, k, v = sets[layer]
                out = fused_attention_gqa_v4(q, k, v, scale=scale, prefix_len=shape.P)
        return out

    # capture the chunk in a CUDA graph (warm the op on a side stream first)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chunk()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = chunk()
    gathered = torch.empty((GLOBAL_B,) + tuple(static_out.shape[1:]), device="cuda",
                           dtype=static_out.dtype) if world > 1 else None

    def step():
        graph.replay()
        if world > 1:
            # outputs gathered over NVLink; shards are equal when world | 2048
            dist.all_gather_into_tensor(gathered, static_out)

    for _ in range(args.warmup):
        step()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    stream = torch.cuda.current_stream()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    barrier(world)
    clk = clocks.stop()
    ms = max_over_ranks(t0.elapsed_time(t1), world)
    ms_per_step = ms / args.steps
    calls_per_s = CALLS_PER_STEP * args.steps / (ms / 1e3)

    # kernel-only timing of the attention launches (no all-gather), for the roofline
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    reps = max(2, args.steps // 2)
    barrier(world)
    k0.record(stream)
    for _ in range(reps):
        graph.replay()
    k1.record(stream)
    torch.cuda.synchronize()
    launch_s = k0.elapsed_time(k1) / 1e3 / (reps * CALLS_PER_STEP)
    launch_s = max_over_ranks(launch_s, world)

    peaks, peak_src = load_peaks()
    bytes_per_launch = wl.attn_bytes(shape)
    flops_per_launch = wl.attn_flops(shape)
    achieved_gbs = bytes_per_launch / launch_s / 1e9
    achieved_tflops = flops_per_launch / launch_s / 1e12
    traffic = attention_traffic(B)
    roofline = {
        "bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peaks["hbm_gbs"],
        "unit": "GB/s", "frac": round(achieved_gbs / peaks["hbm_gbs"], 4),
        "traffic": traffic,
        "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum, median of the launches "
                          f"in {os.path.relpath(NCU_ATTN_CSV, REPO)} (B={NCU_ATTN_BATCH}) scaled to "
                          f"B={B}", "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"
        if peak_src == "measured" else "fallback 6.65 TB/s",
        "kernel": "gqa_attention_sm100", "us_per_launch": round(launch_s * 1e6, 3),
        "algorithmic_bytes_per_launch": bytes_per_launch,
        "tensor_tflops": round(achieved_tflops, 1),
        "tensor_frac": round(achieved_tflops / peaks["bf16_tflops"], 4),
        "flops_per_launch": flops_per_launch,
    }

    # e2e: through the torch op with pinned host buffers, copies timed
    e2e = bench_e2e(args, rank, world, shape, lo)

    line = {
        "metric": METRIC, "value": round(calls_per_s, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "us_per_call": round(1e6 / calls_per_s, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v of the SmolVLA expert shapes)",
        "config": {"workload": C5_WORKLOAD,
                   "global_batch": GLOBAL_B, "per_gpu_batch": B, "calls_per_step": CALLS_PER_STEP,
                   "parallelism": f"batch-shard x{world}",
                   "l2": "inputs > L2: 16 rotating per-layer input sets, >=144 MB each",
                   "cuda_graph": True},
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": CALLS_PER_STEP * args.steps * world,
        "clocks": clk,
    }
    if world > 1:
        dist.barrier()
    del graph
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(target_s=args.cpu_seconds)
    if rank == 0 and world == 1 and not args.no_softmax:
        line["softmax"] = bench_softmax()
    if rank == 0 and world == 1 and not args.no_sites:
        line["sites"] = bench_sites()
    if rank == 0 and world == 1 and not args.no_comparators:
        line["comparators"] = bench_comparators()
    return line


def bench_e2e(args, rank, world, shape, lo):
    """End to end through the public op with host buffers, as a serving loop
    runs it: each step copies its q/k/v from pinned host memory, calls
    torch.ops.vlak.fused_attention_gqa_v4 and copies o back to pinned host
    memory. Uploads, calls and downloads run on three streams with two device
    input sets, so step i+1's upload overlaps step i's call and download
    (host->device and device->host use the link in opposite directions)."""
    from kernels.attention import fused_attention_gqa_v4

    q, k, v = wl.attn_inputs(shape, seed=lo)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    dev = [tuple(torch.empty_like(t) for t in (q, k, v)) for _ in range(2)]
    del q, k, v
    steps = max(3, args.steps // 2)
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def step(i):
        b = i % 2
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(computed[b])  # step i-2's call has read these inputs
            for d, h in zip(dev[b], (hq, hk, hv)):
                d.copy_(h, non_blocking=True)
            uploaded[b].record(up)
        comp.wait_event(uploaded[b])
        o = fused_attention_gqa_v4(*dev[b], scale=0.125, prefix_len=shape.P)
        computed[b].record(comp)
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            ho.copy_(o, non_blocking=True)
            o.record_stream(down)

    def run(n):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(comp)
        up.wait_event(start)
        down.wait_event(start)
        for i in range(n):
            step(i)
        comp.wait_stream(up)
        comp.wait_stream(down)
        end.record(comp)
        torch.cuda.synchronize()
        return start.elapsed_time(end)

    run(2)
    barrier(world)
    ms = max_over_ranks(run(steps), world)
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2 * world
    d2h = ho.numel() * 2 * world
    return {"value": round(steps / (ms / 1e3), 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "note": "one call per step through torch.ops.vlak.fused_attention_gqa_v4 with "
                    "pinned host q/k/v copied in and o copied out inside the timed region; "
                    "uploads, calls and downloads pipelined on three streams"}


def time_calls(fn, calls: int, warmup: int = 5) -> float:
    """Mean seconds per call of fn() over `calls` back-to-back launches."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(calls):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / calls


def time_graph(fns, replays: int = 5) -> float:
    """Mean seconds per call of the calls fns (each a zero-argument launch)
    captured once into a CUDA graph and replayed: device time without the
    host's per-call dispatch."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for f in fns[:3]:
            f()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in fns:
            f()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / 1e3 / (replays * len(fns))


def bench_sites():
    """Per-call times of the other attention sites on one GPU (reported, not
    the headline): C3 expert self-attention at B = 1, 8, 64, C4 prefix
    attention with per-sample lengths at B = 1, 16, 128, and the SigLIP
    vision site (1, 12, 1024, 64) through vlak::fused_attention beside torch
    SDPA. Inputs rotate over enough sets to exceed L2 where a call is small.
    "us" is eager (each call dispatched from Python, host overhead included
    when the kernel is shorter than the dispatch); "graph_us" replays the same
    calls from a CUDA graph (device time)."""
    import torch.nn.functional as F

    from kernels.attention import (fused_attention, fused_attention_gqa_v4,
                                   fused_attention_gqa_varlen)

    peaks, _ = load_peaks()
    res = {}
    for B in (1, 8, 64):
        s = wl.expert_shape(B)
        nsets = max(1, min(64, (256 << 20) // wl.attn_bytes(s)))
        sets = [wl.attn_inputs(s, seed=10 + i) for i in range(nsets)]
        it = [0]

        def call():
            q, k, v = sets[it[0] % nsets]
            it[0] += 1
            fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=s.P)

        t = time_calls(call, 200)
        tg = time_graph([lambda i=i: fused_attention_gqa_v4(*sets[i % nsets], scale=0.125,
                                                             prefix_len=s.P) for i in range(32)])
        res[f"C3_B{B}"] = {"us": round(t * 1e6, 2), "graph_us": round(tg * 1e6, 2),
                           "GB/s": round(wl.attn_bytes(s) / t / 1e9, 1),
                           "TFLOP/s": round(wl.attn_flops(s) / t / 1e12, 2),
                           "tensor_frac": round(wl.attn_flops(s) / t / 1e12 / peaks["bf16_tflops"], 4),
                           "input_sets": nsets}
        del sets
    for B in (1, 16, 128):
        s = wl.prefix_shape(B)
        nsets = max(1, min(32, (256 << 20) // wl.attn_bytes(s)))
        sets = [wl.attn_inputs(s, seed=20 + i) for i in range(nsets)]
        L = wl.c4_lengths(B, seed=B)
        it = [0]

        def call():
            q, k, v = sets[it[0] % nsets]
            it[0] += 1
            fused_attention_gqa_varlen(q, k, v, L)

        t = time_calls(call, 100)
        tg = time_graph([lambda i=i: fused_attention_gqa_varlen(*sets[i % nsets], L)
                         for i in range(32)])
        res[f"C4_varlen_B{B}"] = {"us": round(t * 1e6, 2), "graph_us": round(tg * 1e6, 2),
                                  "GB/s": round(wl.attn_bytes(s) / t / 1e9, 1),
                                  "TFLOP/s": round(wl.varlen_flops(L) / t / 1e12, 2),
                                  "input_sets": nsets}
        del sets
    q, k, v = wl.siglip_inputs()
    flops = 4 * 64 * 12 * 1024 * 1024
    t_ours = time_calls(lambda: fused_attention(q, k, v), 100)
    t_sdpa = time_calls(lambda: F.scaled_dot_product_attention(q, k, v), 100)
    g_ours = time_graph([lambda: fused_attention(q, k, v)] * 32)
    g_sdpa = time_graph([lambda: F.scaled_dot_product_attention(q, k, v)] * 32)
    res["SigLIP_1x12x1024"] = {"us": round(t_ours * 1e6, 2), "graph_us": round(g_ours * 1e6, 2),
                               "TFLOP/s": round(flops / g_ours / 1e12, 1),
                               "torch_sdpa_us": round(t_sdpa * 1e6, 2),
                               "torch_sdpa_graph_us": round(g_sdpa * 1e6, 2)}
    return res


def time_flushed(fn, iters: int = 10) -> float:
    """Median seconds of fn() with L2 flushed before every call: a 256 MB
    write (larger than the 126 MB L2), then a 256 MB read of another buffer,
    so the timed kernel starts with a cold L2 that holds no dirty lines (their
    write-back would otherwise be charged to it)."""
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")
    clean = torch.ones(64 * 2**20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    for _ in range(3):
        fn()
    times = []
    for _ in range(iters):
        flush.zero_()
        torch.sum(clean, dim=0, out=sink)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    del flush, clean
    return statistics.median(times)


def time_softmax_flushed(x, iters: int = 10) -> float:
    """time_flushed of softmax(x, "auto")."""
    from kernels.softmax import softmax

    return time_flushed(lambda: softmax(x, "auto"), iters)


def bench_softmax():
    """C2 bf16 softmax over its whole grid (rows {256, 1024, 8192} x cols {241,
    1024, 4096, 16384, 32768} and the narrow [983040, 291]) and C1 fp32
    [4096, 1024], 1 GPU, L2 flushed before every call. The 8192 x 32768 line
    is the headline; cases below ~1 MB are launch-bound and reported only."""
    from kernels.softmax import _auto_version

    peaks, _ = load_peaks()
    res = {}

    def one(name, x):
        t = time_softmax_flushed(x)
        nbytes = wl.softmax_bytes(x.shape[0], x.shape[1], x.element_size())
        gbs = nbytes / t / 1e9
        res[name] = {"us": round(t * 1e6, 2), "GB/s": round(gbs, 1),
                     "frac_hbm": round(gbs / peaks["hbm_gbs"], 4),
                     "l2": "flushed (256 MB write, then 256 MB clean read)",
                     "version": _auto_version(x)}

    one("C2_bf16_8192x32768", wl.softmax_c2(8192, 32768))
    one("C1_fp32_4096x1024", wl.softmax_c1())
    grid = {}
    for rows in wl.C2_ROWS:
        for cols in wl.C2_COLS:
            if (rows, cols) == (8192, 32768):
                continue
            one(f"C2_{rows}x{cols}", wl.softmax_c2(rows, cols))
    one(f"C2_narrow_{wl.C2_NARROW[0]}x{wl.C2_NARROW[1]}", wl.softmax_c2(*wl.C2_NARROW))
    return res


REF_KERNELS = os.path.join(REPO, "baseline", "_ref", "kernels_sm100a")
SOFTMAX_CMP_CASES = [("C1_fp32_4096x1024", None), ("C2_1024x4096", (1024, 4096)),
                     ("C2_8192x4096", (8192, 4096)), ("C2_1024x16384", (1024, 16384)),
                     ("C2_8192x16384", (8192, 16384)), ("C2_1024x32768", (1024, 32768)),
                     ("C2_8192x32768", (8192, 32768)),
                     (f"C2_narrow_{wl.C2_NARROW[0]}x{wl.C2_NARROW[1]}", wl.C2_NARROW)]


def _softmax_case(shape):
    return wl.softmax_c1() if shape is None else wl.softmax_c2(*shape)


def sdpa_gqa_call(q, k, v, mask):
    """torch SDPA on the op's (B, M, H, 64) / (B, N, Hkv, 64) tensors: views
    to (B, H, M, 64), torch's own GQA (enable_gqa) and the analytic mask as a
    (1, 1, M, N) bool tensor."""
    import torch.nn.functional as F

    return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                          attn_mask=mask, scale=0.125, enable_gqa=True)


def expert_mask(s, device="cuda"):
    r = torch.arange(s.M, device=device)[:, None]
    c = torch.arange(s.N, device=device)[None, :]
    vis = torch.where(c < s.P, (c < s.ds) | (c >= s.de), c <= (s.N - s.M) + r)
    return vis[None, None]


def bench_comparators() -> dict:
    """Bars measured on the same GPU in the same run, reported beside the
    headline and not the target: torch.softmax, cuDNN and CUB softmax over
    C1 / the wide and narrow C2 cases (L2 flushed, as the softmax lines);
    torch SDPA (its own GQA, bool mask) at C3 B=64 and C5 B=2048; the
    L2-warm roof of C3 B=64 (one input set replayed, our kernel); and the
    reference's own kernels rebuilt for sm_100a, timed in a separate process
    (their op schemas collide with ours in one process)."""
    from kernels.attention import fused_attention_gqa_v4
    from kernels.softmax import softmax_cub, softmax_cudnn

    peaks, _ = load_peaks()
    res = {"note": "same-GPU bars, reported only"}
    sm = {}
    for name, shape in SOFTMAX_CMP_CASES:
        x = _softmax_case(shape)
        nbytes = wl.softmax_bytes(x.shape[0], x.shape[1], x.element_size())
        row = {}
        for label, fn in (("torch_softmax", lambda: torch.softmax(x, dim=-1)),
                          ("cudnn", lambda: softmax_cudnn(x)), ("cub", lambda: softmax_cub(x))):
            try:
                t = time_flushed(fn)
                row[label] = {"us": round(t * 1e6, 2),
                              "frac_hbm": round(nbytes / t / 1e9 / peaks["hbm_gbs"], 4)}
            except RuntimeError as e:
                row[label] = {"error": str(e)[:200]}
        sm[name] = row
        del x
    res["softmax"] = sm

    att = {}
    for B in (64, 2048):
        s = wl.expert_shape(B)
        nsets = max(2, min(16, (512 << 20) // wl.attn_bytes(s)))
        sets = [wl.attn_inputs(s, seed=40 + i) for i in range(nsets)]
        mask = expert_mask(s)
        it = [0]

        def sdpa():
            q, k, v = sets[it[0] % nsets]
            it[0] += 1
            return sdpa_gqa_call(q, k, v, mask)

        row = {"input_sets": nsets}
        try:
            t = time_calls(sdpa, 20 if B == 2048 else 100)
            row["torch_sdpa_us"] = round(t * 1e6, 2)
            row["torch_sdpa_frac_hbm"] = round(wl.attn_bytes(s) / t / 1e9 / peaks["hbm_gbs"], 4)
        except RuntimeError as e:
            row["torch_sdpa_error"] = str(e)[:200]
        it[0] = 0

        def ours():
            q, k, v = sets[it[0] % nsets]
            it[0] += 1
            return fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=s.P)

        t = time_calls(ours, 20 if B == 2048 else 100)
        row["ours_us"] = round(t * 1e6, 2)
        att[f"C3_B{B}" if B == 64 else "C5_B2048_one_call"] = row
        del sets
    # the L2-warm roof: one C3 B=64 input set (36 MB) replayed from a graph
    s = wl.expert_shape(64)
    q, k, v = wl.attn_inputs(s, seed=7)
    tw = time_graph([lambda: fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=s.P)] * 32, 10)
    att["C3_B64_l2_warm"] = {"graph_us": round(tw * 1e6, 2),
                             "TFLOP/s": round(wl.attn_flops(s) / tw / 1e12, 1),
                             "tensor_frac": round(wl.attn_flops(s) / tw / 1e12 / peaks["bf16_tflops"], 4),
                             "note": "one 36 MB input set replayed: K/V/Q stay in L2"}
    res["attention"] = att
    res["reference_kernels_sm100a"] = run_ref_kernels_worker()
    return res


def run_ref_kernels_worker(timeout_s: int = 300) -> dict:
    """Times the reference's own kernels (rebuilt for sm_100a by
    baseline/build_ref_kernels.py) in a child process."""
    if not os.path.exists(os.path.join(REF_KERNELS, "manifest.json")):
        return {"unavailable": "not built (baseline/build_ref_kernels.py needs a reference checkout)"}
    try:
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--ref-kernels-worker"],
                           capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"worker exceeded {timeout_s} s"}
    for line in reversed(r.stdout.splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    return {"unavailable": f"worker rc {r.returncode}: {r.stderr.strip()[-300:]}"}


def ref_kernels_worker():
    """Child process: loads the reference's kernels (their own torch.ops.vlak
    registrations; this package's libraries are not loaded here) and times
    softmax versions 1 and 4 on the softmax comparator cases, and the v3 / v4
    GQA attention at C3 B = 1, 8, 64 (graph replay) and one C5 B=2048 call.
    A C3 B=8 call is checked against torch SDPA in fp32 (max abs error)."""
    torch.cuda.set_device(0)
    man = json.load(open(os.path.join(REF_KERNELS, "manifest.json")))
    out = {"build": "reference sources unmodified, nvcc -O3 --use_fast_math -gencode "
                    "arch=compute_100a,code=sm_100a (baseline/build_ref_kernels.py)"}
    loaded = []
    for name, st in man.items():
        if st.get("ok"):
            torch.ops.load_library(os.path.join(REF_KERNELS, st["so"]))
            loaded.append(name)
        else:
            out[name] = {"unavailable": st.get("error", "not built")}
    out["loaded"] = loaded
    peaks, _ = load_peaks()
    if "vlak_ref_softmax" in loaded:
        sm = {}
        for name, shape in SOFTMAX_CMP_CASES:
            x = _softmax_case(shape)
            nbytes = wl.softmax_bytes(x.shape[0], x.shape[1], x.element_size())
            row = {}
            for ver in (1, 4):
                t = time_flushed(lambda: torch.ops.vlak.softmax(x, ver))
                row[f"v{ver}"] = {"us": round(t * 1e6, 2),
                                  "frac_hbm": round(nbytes / t / 1e9 / peaks["hbm_gbs"], 4)}
            sm[name] = row
            del x
        out["softmax"] = sm
    ops = []
    if "vlak_ref_attention" in loaded:
        ops.append(("v3", torch.ops.vlak.fused_attention_gqa))
    if "vlak_ref_attention_v4" in loaded:
        ops.append(("v4", torch.ops.vlak.fused_attention_gqa_v4))
    att = {}
    for B in (1, 8, 64):
        s = wl.expert_shape(B)
        nsets = max(1, min(64, (256 << 20) // wl.attn_bytes(s)))
        sets = [wl.attn_inputs(s, seed=10 + i) for i in range(nsets)]
        row = {"input_sets": nsets}
        for label, op in ops:
            tg = time_graph([lambda i=i, op=op: op(*sets[i % nsets], 0.125, s.P, 0, 0)
                             for i in range(32)])
            row[f"{label}_graph_us"] = round(tg * 1e6, 2)
        if B == 8:
            q, k, v = sets[0]
            ref = sdpa_gqa_call(q.float(), k.float(), v.float(), expert_mask(s))
            for label, op in ops:
                got = op(q, k, v, 0.125, s.P, 0, 0).float().transpose(1, 2)
                row[f"{label}_max_abs_err_vs_fp32_sdpa"] = float((got - ref).abs().max())
        att[f"C3_B{B}"] = row
        del sets
    s = wl.expert_shape(2048)
    sets = [wl.attn_inputs(s, seed=60 + i) for i in range(2)]
    row = {}
    for label, op in ops:
        it = [0]

        def call(op=op):
            q, k, v = sets[it[0] % 2]
            it[0] += 1
            op(q, k, v, 0.125, s.P, 0, 0)

        t = time_calls(call, 10, warmup=2)
        row[f"{label}_us"] = round(t * 1e6, 2)
        row[f"{label}_frac_hbm"] = round(wl.attn_bytes(s) / t / 1e9 / peaks["hbm_gbs"], 4)
    att["C5_B2048_one_call"] = row
    out["attention"] = att
    print(json.dumps(out), flush=True)


def cpu_baseline_sample(target_s: float = 10.0) -> dict:
    """The oracle port of the reference's CPU path (torch SDPA, fp32, all host
    threads) on the C5 call itself: whole B=2048 calls, as many as fit in
    ~target_s after one untimed call."""
    from oracle import gqa_attention_torch_cpu

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    s = wl.expert_shape(GLOBAL_B)
    q, k, v = wl.attn_inputs(s, device="cpu", seed=5)
    gqa_attention_torch_cpu(q, k, v, s.P, scale=0.125)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < target_s or n < 2:
        gqa_attention_torch_cpu(q, k, v, s.P, scale=0.125)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} whole C5 calls (B=2048 expert self-attn), torch SDPA fp32 with "
                      f"bool mask and repeat_interleave GQA on host, {dt:.1f} s"}


# ---------------------------------------------------------------- reference arm

def bench_reference(args, rank, world):
    """The reference's CPU path (torch SDPA with bool mask + repeat_interleave
    GQA, fp32, all host threads) on the same C5 call, rank 0 only: each step
    is one whole B=2048 call (the unit of the metric), W untimed then K timed."""
    if rank != 0:
        return None
    from oracle import gqa_attention_torch_cpu

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    s = wl.expert_shape(GLOBAL_B)
    q, k, v = wl.attn_inputs(s, device="cpu", seed=5)
    for _ in range(max(1, args.warmup)):
        gqa_attention_torch_cpu(q, k, v, s.P, scale=0.125)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        gqa_attention_torch_cpu(q, k, v, s.P, scale=0.125)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/k/v of the SmolVLA expert shapes)",
        "config": {"workload": C5_WORKLOAD, "global_batch": GLOBAL_B,
                   "step": "one whole B=2048 call per step",
                   "parallelism": f"host CPU, {threads} threads (the reference has no sm_100 "
                                  "code; its CPU path is torch)"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.steps} whole C5 calls (B=2048), torch SDPA fp32"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------- profiling mode

def profile_case(args):
    """A few eager launches of one kernel on a small case (for ncu captures):
    attention at C3/C5 shapes with --batch queries, or softmax --rows x --cols
    bf16. Inputs of both exceed L2 at the default sizes."""
    torch.cuda.set_device(0)
    if args.case == "attn":
        from kernels.attention import fused_attention_gqa_v4

        s = wl.expert_shape(args.batch)
        sets = [wl.attn_inputs(s, seed=i) for i in range(2)]
        for i in range(args.calls):
            q, k, v = sets[i % 2]
            fused_attention_gqa_v4(q, k, v, scale=0.125, prefix_len=s.P)
    else:
        from kernels.softmax import softmax

        x = wl.softmax_c2(args.rows, args.cols)
        for _ in range(args.calls):
            softmax(x, "auto")
    torch.cuda.synchronize()
    print(f"profile case {args.case} done")


# ---------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-softmax", action="store_true")
    ap.add_argument("--no-sites", action="store_true",
                    help="skip the per-site attention timings (C3, C4, SigLIP)")
    ap.add_argument("--no-comparators", action="store_true",
                    help="skip the same-GPU bars (torch, cuDNN, CUB, reference kernels)")
    ap.add_argument("--ref-kernels-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--case", choices=["attn", "softmax"], default=None,
                    help="profiling mode: a few eager calls of one kernel, no JSON line")
    ap.add_argument("--batch", type=int, default=512)
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--cols", type=int, default=32768)
    ap.add_argument("--calls", type=int, default=4)
    args = ap.parse_args()

    if args.ref_kernels_worker:
        ref_kernels_worker()
        return
    if args.case is not None:
        profile_case(args)
        return

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = bench_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    rank, world, local = dist_setup(args.gpus)
    try:
        line = bench_ours(args, rank, world, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
