#!/usr/bin/env python
"""Benchmark of the B200 block-local attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5] [--halo 1]
    python bench.py --impl reference ...      # the reference's CPU algorithm

A step is one forward pass of block-local attention over one batch of the
workload.  The default is c5, the configuration the headline metric is
quoted on: batch 256, 16 heads, seq 8192, head_dim 64, block 128, Block3 =
halo 1, valid lengths U[4096, 8192], N(0,1) inputs from seed 4 (34.4 GB of
q, k, v and out, generated on the device).

Under torchrun (N ranks, one per GPU) the workload's batch x heads slices are
split over the ranks by raya_attn_shard, balanced by allowed pairs, and each
rank generates and runs only its own slices (strong scaling; no collective
in the timed region).  `value` is whole-job algorithmic GFLOP/s (4 * head_dim
FLOPs per allowed query/key pair, counted exactly), timed with CUDA events
over K steps, max over ranks.  `gather` times, separately, the output gather
to rank 0 over NVLink and checks it bit for bit.  `e2e` is the same metric
through the host-buffer API (raya_attn_forward_host: pinned host inputs ->
device -> kernel -> host output, synchronous), every rank on its own slices,
wall clock, max over ranks.  `--scaling weak` gives every rank a whole batch
of the workload instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 2**20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="c5")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the workload's slices split over the ranks; weak: a whole batch per rank")
    ap.add_argument("--no-gather", action="store_true", help="skip the timed output gather to rank 0 (N > 1)")
    ap.add_argument("--gather-reps", type=int, default=3)
    ap.add_argument("--halo", type=int, default=1)
    ap.add_argument("--kernel", type=int, default=0, help="0 auto, 1 tiled64, 2 rowwise, 34 tc32_ws, 37 tc32_ws two-tile (3xTF32 tensor cores), "
                    "40 tc16_ws, 41 tc16_ws two-tile (3xFP16 tensor cores)")
    ap.add_argument("--e2e-steps", type=int, default=3,
                    help="timed host-buffer calls (each copies the step's inputs in and its output out)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target CPU work of the cpu_baseline sample")
    ap.add_argument("--packed", action="store_true",
                    help="the caller's layout: packed qkv [B][L][3][H][64] in, context [B][L][H][64] out")
    ap.add_argument("--rope-theta", type=float, default=0.0,
                    help="with --packed: raya's rotary embedding on q and k (0 = off)")
    ap.add_argument("--raya-bench", action="store_true",
                    help="run raya's local_attention bench shapes and write results/kernel-bench/*.json")
    ap.add_argument("--soak", type=float, default=1.0,
                    help="seconds of untimed steps, clock-sampled, right before the timed region")
    args = ap.parse_args()
    if args.packed and args.kernel != 0:
        ap.error("--kernel does not apply with --packed: the packed entry points choose their kernel "
                 "(raya_attn_kernel_for with packed != 0)")
    return args


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.gpu_ids = gpu_ids
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", ",".join(str(g) for g in self.gpu_ids)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons),
                "window": "1 s soak of the same step + the timed region, 50 ms period"}


# Used only when MEASURED_PEAKS.json is absent: an earlier measurement of
# this pool's B200s (STREAM-style copy; cuBLAS bf16 GEMM burst).
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks() -> tuple[dict, str]:
    """(peaks, "measured" | "fallback")."""
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(key: str):
    """DRAM bytes per launch from a committed ncu summary, if any."""
    try:
        t = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        return t.get(key)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- reference arm

def run_reference(args) -> None:
    """The reference's algorithm on the host cores: the C restatement of
    raya's Tiled kernel with its AVX2+FMA micro-kernels (oracle/tiled.c), all
    host threads, on the workload of the B200 arm.  The reference itself is
    Rust and cannot be built here (no cargo/rustc)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    from raya_b200.workloads import CONFIGS

    w = CONFIGS[args.workload].with_halo(args.halo)
    threads = host_threads()
    valid = w.valid_len()
    p = oracle.Problem(w.batch, w.heads, w.seq, w.head_dim, mask=oracle.MASK_BLOCK,
                       block=w.block, halo=w.halo)
    # Bounded sample of the workload: whole (batch entry) slices, sized so a
    # step is ~2 s at an assumed 100 GFLOP/s; inputs N(0, stddev^2) on the host.
    pairs_all, _ = oracle.count(p, valid)
    per_b = pairs_all / w.batch * 4 * w.head_dim
    nb = max(1, min(w.batch, int(2.0 * 100e9 / max(per_b, 1.0))))
    ps = oracle.Problem(nb, w.heads, w.seq, w.head_dim, mask=oracle.MASK_BLOCK, block=w.block,
                        halo=w.halo)
    rng = np.random.default_rng(w.seed)
    q, k, v = (rng.standard_normal(ps.numel, dtype=np.float32) * np.float32(w.stddev) for _ in range(3))
    out = np.zeros(ps.numel, dtype=np.float32)
    vs = valid[:nb]
    pairs, rows = oracle.count(ps, vs)
    for _ in range(args.warmup):
        oracle.tiled(ps, q, k, v, vs, threads=threads, out=out)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.tiled(ps, q, k, v, vs, threads=threads, out=out)
    dt = (time.perf_counter() - t0) / args.steps
    gflops = 4 * w.head_dim * pairs / dt / 1e9
    sample = (f"{nb} of {w.batch} sequences x {w.heads} heads of {w.name} (halo {w.halo}) per step, "
              f"N(0,{w.stddev}^2) host inputs")
    line = {
        "metric": "block-local attn GFLOP/s", "value": round(gflops, 3), "unit": "GFLOP/s",
        "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(w, world, args.scaling),
        "queries_per_s": round(rows / dt, 1),
        "cpu_baseline": {"value": round(gflops, 3), "unit": "GFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample, "cpu": cpu_model(),
                         "what": "C restatement of raya Tiled + AVX2 micro-kernels (oracle/tiled.c)"},
        "e2e": {"value": round(gflops, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(w, world: int, scaling: str) -> dict:
    strong = scaling == "strong"
    gb = w.batch if strong else w.batch * world
    per = "" if strong else "/GPU"
    return {"workload": f"{w.name}: batch {w.batch}{per} x {w.heads} heads x seq {w.seq} x d {w.head_dim},"
                        f" block {w.block}, halo {w.halo} ({'Block3' if w.halo == 1 else 'own block'}),"
                        f" valid {w.valid or 'full'}, seed {w.seed}, N(0,{w.stddev}^2)"
                        + (f", {w.layers} layers" if w.layers > 1 else ""),
            "global_batch": gb, "seq_len": w.seq, "heads": w.heads,
            "head_dim": w.head_dim, "block": w.block, "halo": w.halo,
            "parallelism": (f"batch x heads slices split over {world} GPU(s) by allowed pairs "
                            "(raya_attn_shard), no collective in the timed region" if strong else
                            f"a whole batch per GPU on {world} GPU(s), no collective"),
            "l2": l2_note(4 * w.numel * 4 / (world if strong else 1))}


def l2_note(nbytes: float) -> str:
    mib = nbytes / 2**20
    if nbytes > L2_BYTES:
        return f"inputs+output {mib:.0f} MiB per GPU > 126 MiB L2 (no flush needed)"
    return f"inputs+output {mib:.0f} MiB per GPU fit in the 126 MiB L2 (not flushed: L2-resident between steps)"


# ---------------------------------------------------------------- B200 arm

def kernel_label(rb, chosen, shape, packed, block) -> str:
    # (the row tiles per CTA of kernel 37 follow raya_attn.cu's rule)
    if chosen == rb.KERNEL_ROWWISE:
        return "rowwise (raya_b200/csrc/rowwise.cuh)"
    if chosen == rb.KERNEL_TC32_WS:
        return ("tc32_ws, two MMA-issuing warps, PV summed in fp32 registers, 3xTF32 tcgen05 "
                "(raya_b200/csrc/tc32_ws.cuh), kernel id 34")
    if chosen == rb.KERNEL_TC32_WS2:
        tiles = (shape.seq + 127) // 128
        many = tiles % 4 == 0 and block >= 128 and shape.batch * shape.heads * tiles >= 16384
        units = "four 128-row tiles (a whole slice)" if tiles == 4 else "four 128-row tiles" if many else "two 128-row tiles"
        return (f"tc32_ws with {'two 128-row tiles' if packed else units} per CTA"
                + " (raya_b200/csrc/tc32_ws.cuh), kernel id 37")
    if chosen == rb.KERNEL_TC16_WS:
        return ("tc16_ws, 3xFP16 tcgen05 kind::f16 with power-of-two operand scaling, two MMA-issuing warps, "
                "PV summed in fp32 registers (raya_b200/csrc/tc16_ws.cuh), kernel id 40")
    if chosen == rb.KERNEL_TC16_WS2:
        return ("tc16_ws persistent (one CTA per SM walking its 128-row tiles), 3xFP16 tcgen05 kind::f16 "
                "(raya_b200/csrc/tc16_ws.cuh), kernel id 41")
    return f"tiled64 (raya_b200/csrc/tiled64.cuh), kernel id {chosen}"


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    import raya_b200 as rb
    from raya_b200 import shards
    from raya_b200.workloads import CONFIGS, fill_device

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    w = CONFIGS[args.workload].with_halo(args.halo)
    D = w.head_dim
    strong = args.scaling == "strong"
    # The global problem and this rank's part of it.  Strong scaling: the
    # workload's batch x heads slices are split over the ranks by
    # raya_attn_shard (balanced by allowed pairs), each rank generating only
    # its own slices (inputs are a function of the global element index).
    # Weak scaling: every rank runs a whole batch of the workload (entries
    # rank*batch ..), as independent problems.
    gbatch = w.batch if strong else w.batch * world
    gvalid = w.valid_len(first=0, count=gbatch)
    gshape = rb.AttnShape(heads=w.heads, seq=w.seq, head_dim=D, batch=gbatch)
    gparams = rb.AttnParams.new(rb.Mask.block(w.halo), gvalid, D, block=w.block)
    sp = shards.plan(gshape, gparams, world) if strong else None
    if strong:
        bh0, bh1 = sp.range(rank)
        shape, params = shards.shard_problem(gshape, gparams, bh0, bh1)
        valid = np.asarray(params.valid_len, dtype=np.int32)
    else:
        bh0, bh1 = rank * w.batch * w.heads, (rank + 1) * w.batch * w.heads
        valid = gvalid[rank * w.batch:(rank + 1) * w.batch]
        shape = rb.AttnShape(heads=w.heads, seq=w.seq, head_dim=D, batch=w.batch)
        params = rb.AttnParams.new(rb.Mask.block(w.halo), valid, D, block=w.block)
    pairs, rows = rb.work(shape, params) if shape.batch > 0 else (0, 0)
    slice_elems = w.seq * D
    n = (bh1 - bh0) * slice_elems
    gather_on = strong and world > 1 and not args.no_gather
    # One (q, k, v, out) set per encoder layer (c4 has 12; the others 1).
    # Rank 0 of a gathered run owns the whole output tensor of layer 0 and
    # writes its own slices straight into it.
    layers = []
    for layer in range(w.layers):
        t = [torch.empty(max(n, 1), dtype=torch.float32, device=dev) for _ in range(3)]
        fill_device(w, t, layer=layer, bh0=bh0)
        if gather_on and rank == 0 and layer == 0:
            full = torch.empty(sp.ranges[-1][1] * slice_elems, dtype=torch.float32, device=dev)
            t.append(full[bh0 * slice_elems:bh1 * slice_elems])
        else:
            t.append(torch.empty(max(n, 1), dtype=torch.float32, device=dev))
        layers.append(tuple(t))
    q, k, v, out = layers[0]
    pairs, rows = pairs * w.layers, rows * w.layers
    dvalid = torch.from_numpy(valid).to(dev) if shape.batch > 0 else None
    kern = rb.Cuda(rb.CudaConfig(device=local, kernel=args.kernel))
    chosen = (rb.kernel_for(shape, params, packed=args.packed, rope=args.rope_theta > 0)
              if args.kernel == rb.KERNEL_AUTO else args.kernel) if shape.batch > 0 else rb.KERNEL_AUTO
    tiled_ids = set(rb._lib.KERNEL_TILED64_VARIANTS.values()) | {rb.KERNEL_TILED64}
    F16_KERNELS = (rb.KERNEL_TC16_WS, rb.KERNEL_TC16_WS2)
    TENSOR_KERNELS = (rb.KERNEL_TC32_WS, rb.KERNEL_TC32_WS2) + F16_KERNELS
    stream = torch.cuda.current_stream(dev)

    # Live FFMA peak of this GPU (the fp32-equivalent denominator: no FP32
    # figure is in MEASURED_PEAKS.json), measured before the timed region.
    ffma_tflops = rb.ffma_peak(5)

    if args.packed:
        # The same numbers laid out as the encoder's packed projection.
        packed = []
        for lq, lk, lv, lo in layers:
            qkv = torch.stack([t.view(shape.batch, shape.heads, w.seq, D).transpose(1, 2) for t in (lq, lk, lv)],
                              dim=2).contiguous().view(-1)
            packed.append((qkv, torch.empty_like(lo)))
        ws = torch.empty(w.seq * 64, dtype=torch.float32, device=dev) if args.rope_theta > 0 else None

    def step():
        if shape.batch == 0:
            return
        if args.packed:
            for qkv, ctx in packed:
                kern.attend_packed(shape, params, qkv, ctx, valid_len=dvalid, rope_theta=args.rope_theta or None,
                                   workspace=ws, stream=stream)
            return
        for lq, lk, lv, lo in layers:  # layers back to back on one stream
            kern.attend_device(shape, params, lq, lk, lv, lo, valid_len=dvalid, stream=stream)

    for _ in range(max(args.warmup, 3)):
        step()
    rb.sync_status(stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    # Clocks: nvidia-smi samples every 50 ms from the start of an untimed soak
    # of the same step (about args.soak seconds, so that the samples see the
    # GPU under this load) through the end of the timed region, which follows
    # the soak with no gap.
    sampler = ClockSampler(list(range(world)) if rank == 0 else [local])
    if rank == 0:
        sampler.start()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak:
        for _ in range(4):
            step()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    clocks = sampler.stop() if rank == 0 else None
    rb.sync_status(stream)
    if world > 1:
        t = torch.tensor([ms, float(pairs), float(rows)], dtype=torch.float64, device=dev)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        ms_max, pairs_all, rows_all = float(mx[0]), float(t[1]), float(t[2])
    else:
        ms_max, pairs_all, rows_all = ms, float(pairs), float(rows)
    flops_all = 4.0 * D * pairs_all
    gflops = flops_all / (ms_max * 1e-3) / 1e9
    qps = rows_all / (ms_max * 1e-3)

    # The output gather to rank 0 (strong scaling, N > 1), timed on its own:
    # every rank's layer-0 output into rank 0's whole-output tensor over
    # NVLink.  Then rank 0 checks that gathered slices of every other rank are
    # bit-identical to the same slices run on its own GPU.
    gather = None
    if gather_on:
        reps = max(1, args.gather_reps)
        times = []
        for _ in range(reps + 1):  # the first is a warm-up
            dist.barrier()
            torch.cuda.synchronize(dev)
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            shards.gather_to_rank0(out, sp, rank, out=full if rank == 0 else None)
            g1.record(stream)
            torch.cuda.synchronize(dev)
            times.append(g0.elapsed_time(g1))
        gt = torch.tensor([statistics.median(times[1:])], dtype=torch.float64, device=dev)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        moved = 4 * (sp.ranges[-1][1] - sp.range(0)[1] + sp.range(0)[0]) * slice_elems
        gather = {"ms": round(float(gt[0]), 3), "bytes_to_rank0": moved,
                  "gbps_into_rank0": round(moved / (float(gt[0]) * 1e-3) / 1e9, 1),
                  "how": "NCCL point-to-point receives straight into rank 0's output tensor "
                         "(raya_b200.shards.gather_to_rank0), median of "
                         f"{reps} after a warm-up, CUDA events, max over ranks; not in `value`"}
        if rank == 0:
            gather["check"] = gather_check(rb, w, gshape, gparams, sp, full, dev)

    # Roofline of the kernel (per launch on this rank; a step is w.layers launches).
    flops_launch = 4.0 * D * pairs / w.layers
    bytes_launch = 4.0 * D * (3 * float(valid.sum()) * (1 if strong else w.heads)
                              + shape.batch * shape.heads * w.seq)
    launch_ms = ms / w.layers
    achieved_tf = flops_launch / (launch_ms * 1e-3) / 1e12
    peaks, peak_kind = load_peaks()
    hbm = peaks.get("hbm_gbs")
    tkey = (f"{w.name}-halo{w.halo}" + (f"-k{chosen}" if chosen in TENSOR_KERNELS else "")
            + ("-packed" if args.packed else ""))
    traffic = load_traffic(tkey) if world == 1 else None
    hbm_obj = {"achieved": round(bytes_launch / (launch_ms * 1e-3) / 1e9, 1), "peak": hbm,
               "unit": "GB/s", "frac": round(bytes_launch / (launch_ms * 1e-3) / 1e9 / hbm, 4) if hbm else None,
               "peak_source": f"MEASURED_PEAKS.json hbm_gbs (of {peak_kind})" if peak_kind == "measured"
               else "fallback copy bandwidth of this pool (of fallback)"}
    if chosen in TENSOR_KERNELS:
        # Three tensor-core products per fp32 product (hi*lo, lo*hi, hi*hi):
        # the algorithmic tensor work is 3 x 4 * head_dim per allowed pair.
        # Dense fp16 runs at the bf16 rate, dense TF32 at half of it.
        f16 = chosen in F16_KERNELS
        t_peak = peaks["bf16_tflops"] if f16 else peaks["bf16_tflops"] / 2
        roofline = {"bound": "tensor", "achieved": round(3 * achieved_tf, 3), "peak": round(t_peak, 1),
                    "unit": "TFLOP/s", "frac": round(3 * achieved_tf / t_peak, 4),
                    "peak_source": (f"dense fp16 = bf16_tflops (of {peak_kind})" if f16
                                    else f"dense TF32 = bf16_tflops / 2 (of {peak_kind})"),
                    "work": (f"3 {'fp16' if f16 else 'TF32'} products (hi*lo, lo*hi, hi*hi) x 4 * head_dim "
                             "flops per allowed pair"),
                    "fp32_equivalent": {"achieved": round(achieved_tf, 3), "ffma_peak": round(ffma_tflops, 3),
                                        "frac": round(achieved_tf / ffma_tflops, 4)},
                    "traffic": traffic, "algorithmic_bytes": bytes_launch, "hbm": hbm_obj}
    else:
        roofline = {"bound": "ffma", "achieved": round(achieved_tf, 3), "peak": round(ffma_tflops, 3),
                    "unit": "TFLOP/s", "frac": round(achieved_tf / ffma_tflops, 4),
                    "peak_source": "measured live: raya_attn_ffma_peak (FP32 FFMA probe, this GPU)",
                    "nominal_peak": round(148 * 128 * 2 * 1.965e9 / 1e12, 1),
                    "traffic": traffic, "algorithmic_bytes": bytes_launch, "hbm": hbm_obj}
    if world > 1:
        roofline["per"] = "rank 0's launches"

    # End to end through the host-buffer API (pinned inputs, synchronous), on
    # every rank's own slices at once; the max over ranks is the step time.
    e2e = None
    if not args.no_e2e and not args.packed:
        e2e = run_e2e(args, rb, kern, shape, params, q, k, v, out, valid, w, world, dev, flops_all / w.layers)

    # Stage proportions of one extra, instrumented launch (the reference
    # bench's "stages" field, benches/local_attention.rs:127-130,155-157).
    stages = None
    if not args.packed and shape.batch > 0 and (chosen in tiled_ids or chosen in TENSOR_KERNELS):
        st = rb.stage_times(shape, params, q, k, v, out, valid_len=dvalid, kernel=chosen)
        stages = {key: round(val, 2) for key, val in st.items() if key.endswith("pct")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.packed:
        cpu = cpu_baseline(args, w, q, k, v, out, gvalid if strong else valid, dev)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "block-local attn GFLOP/s", "value": round(gflops, 3), "unit": "GFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), device-generated)",
        "config": workload_config(w, world, args.scaling),
        "queries_per_s": round(qps, 1),
        "frac_fp32_peak": round(achieved_tf / ffma_tflops, 4),
        "gpu_launches": args.steps * w.layers,
        "layout": ("packed qkv -> context" + (f", rope theta {args.rope_theta:g}" if args.rope_theta else "")
                   if args.packed else "head-major q, k, v -> out"),
        "kernel": kernel_label(rb, chosen, shape, args.packed, w.block),
        "kernel_choice": "automatic (raya_attn_kernel_for)" if args.kernel == rb.KERNEL_AUTO else "--kernel",
        "roofline": roofline, "e2e": e2e, "gather": gather, "cpu_baseline": cpu, "clocks": clocks,
        "stages": stages,
    }
    print(json.dumps(line), flush=True)


def gather_check(rb, w, gshape, gparams, sp, full, dev) -> dict:
    """Rank 0: the first and last slice of every rank's range, regenerated
    and run on rank 0's GPU as one call, must equal the gathered output bit
    for bit (slices are independent, so sharding changes no rounding)."""
    import torch

    from raya_b200 import shards

    picks = sorted({x for b, e in sp.ranges if e > b for x in (b, e - 1)})
    n = w.seq * w.head_dim
    tq, tk, tv = (torch.empty(len(picks) * n, dtype=torch.float32, device=dev) for _ in range(3))
    for i, bh in enumerate(picks):
        for t, x in enumerate((tq, tk, tv)):
            rb.fill_normal(x[i * n:(i + 1) * n], w.layer_seed(0), t, bh * n, w.stddev)
    gv = gparams.valid_array(gshape.batch)
    sv = np.array([gv[bh // w.heads] for bh in picks], dtype=np.int32)
    sub_shape = rb.AttnShape(heads=1, seq=w.seq, head_dim=w.head_dim, batch=len(picks))
    sub_params = rb.AttnParams(mask=gparams.mask, block=gparams.block, valid_len=sv, scale=gparams.scale)
    o = torch.empty_like(tq)
    rb.Cuda().attend_device(sub_shape, sub_params, tq, tk, tv, o, valid_len=torch.from_numpy(sv).to(dev))
    rb.sync_status()
    want = torch.cat([full[bh * n:(bh + 1) * n] for bh in picks])
    same = bool(torch.equal(o, want))
    assert same, "gathered slices differ from the same slices run on one GPU"
    return {"slices": picks, "bit_exact": same}


def run_e2e(args, rb, kern, shape, params, q, k, v, out, valid, w, world, dev, flops_step) -> dict | None:
    import torch
    import torch.distributed as dist

    n = shape.numel()
    if n:
        hq, hk, hv, ho = (torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(4))
        for h, d in zip((hq, hk, hv), (q, k, v)):
            h.copy_(d[:n])
        hq_np, hk_np, hv_np, ho_np = (x.numpy() for x in (hq, hk, hv, ho))
        kern.attend(shape, params, hq_np, hk_np, hv_np, ho_np)  # warm-up (staging buffers)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps if n else 0):
        kern.attend(shape, params, hq_np, hk_np, hv_np, ho_np)
    e2e_s = (time.perf_counter() - t0) / args.e2e_steps
    # q, k, v rows below valid_len (the call copies no padding rows) + one length per slice
    h2d = 3 * int(valid.astype(np.int64).sum()) * (shape.heads * w.head_dim * 4) + shape.batch * shape.heads * 4
    d2h = n * 4
    if world > 1:
        t = torch.tensor([e2e_s, float(h2d), float(d2h)], dtype=torch.float64, device=dev)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        e2e_s, h2d_all, d2h_all = float(mx[0]), float(t[1]), float(t[2])
    else:
        h2d_all, d2h_all = float(h2d), float(d2h)
    if n:
        # the host call must agree with the device call (bit for bit when both
        # run the same kernel; --kernel may pick another variant for the device)
        diff = float((ho - out[:n].cpu()).abs().max())
        assert diff < 1e-5 and (args.kernel != 0 or diff == 0.0), \
            f"host-buffer call differs from the device call by {diff}"
    return {"value": round(flops_step / e2e_s / 1e9, 3), "unit": "GFLOP/s",
            "ms_per_step": round(e2e_s * 1e3, 3),
            "h2d_bytes_per_step": int(h2d_all), "d2h_bytes_per_step": int(d2h_all),
            "h2d_gbps": round(h2d_all / e2e_s / 1e9, 1),
            "steps": args.e2e_steps,
            "api": "raya_attn_forward_host (AttentionKernel::attend contract), pinned host buffers, "
                   "every rank its own slices, wall clock, max over ranks"}


def cpu_baseline(args, w, q, k, v, out, valid, dev) -> dict:
    """The oracle's Tiled+AVX2 restatement on the host cores over a bounded
    sample (whole sequences) of the same device-generated inputs.  The
    sample's CPU outputs are also compared with the GPU's outputs for the same
    slices (max-abs 1e-5, the parity bar of the tests)."""
    import oracle

    threads = host_threads()
    D, L, H = w.head_dim, w.seq, w.heads
    # calibrate on one sequence, then size the sample to ~cpu_seconds
    host = {}

    def run(nb):
        ps = oracle.Problem(nb, H, L, D, mask=oracle.MASK_BLOCK, block=w.block, halo=w.halo)
        m = nb * H * L * D
        if host.get("m") != m:
            host.update(m=m, x=tuple(x[:m].cpu().numpy() for x in (q, k, v)))
        qs, ks, vs = host["x"]
        t0 = time.perf_counter()
        o = oracle.tiled(ps, qs, ks, vs, valid[:nb], threads=threads)
        dt = time.perf_counter() - t0
        pairs, _ = oracle.count(ps, valid[:nb])
        return 4 * D * pairs / dt / 1e9, dt, o
    rate, dt1, _ = run(1)
    nb = int(max(1, min(w.batch, args.cpu_seconds / max(dt1, 1e-3))))
    rates, total, reps, o = [], 0.0, 0, None
    while total < args.cpu_seconds and reps < 200:
        rate, dt, o = run(nb)
        rates.append(rate)
        total += dt
        reps += 1
    rate = statistics.median(rates)
    m = nb * H * L * D
    diff = float(np.abs(out[:m].cpu().numpy().astype(np.float64) - o.astype(np.float64)).max())
    return {"value": round(rate, 3), "unit": "GFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{nb} of {w.batch} sequences x {H} heads of {w.name} (same inputs), "
                      f"median of {reps} passes, {total:.1f} s of CPU work",
            "cpu": cpu_model(),
            "what": "C restatement of raya Tiled + AVX2 micro-kernels (oracle/tiled.c)",
            "parity": {"slices": nb * H, "max_abs_vs_gpu": diff, "within_1e-5": diff < 1e-5}}


def raya_bench(args) -> None:
    """raya's local_attention bench on the GPU (raya_b200/kernel_bench.py),
    with the CPU baseline rows of the same file: the Tiled + AVX2 restatement
    at 1 thread and at every host thread, like the reference bench's tiled
    rows (benches/local_attention.rs:114-140)."""
    from raya_b200 import kernel_bench

    threads = host_threads()

    def cpu_rows(seq, mask, q, k, v):
        import oracle

        m = (dict(mask=oracle.MASK_BLOCK, block=128, halo=1) if mask == "block3"
             else dict(mask=oracle.MASK_WINDOW, window=64))
        p = oracle.Problem(1, kernel_bench.HEADS, seq, kernel_bench.HEAD_DIM, **m)
        qh, kh, vh = (x.cpu().numpy() for x in (q, k, v))
        rows = []
        for t in sorted({1, threads}):
            times = []
            for _ in range(3):
                t0 = time.perf_counter()
                oracle.tiled(p, qh, kh, vh, threads=t)
                times.append((time.perf_counter() - t0) * 1e3)
            rows.append({"kernel": "tiled", "mask": mask, "backend": "avx2", "seq": seq,
                         "heads": kernel_bench.HEADS, "head_dim": kernel_bench.HEAD_DIM, "threads": t,
                         "mean_ms": statistics.mean(times), "stddev_ms": statistics.stdev(times),
                         "samples": len(times),
                         "note": "C restatement of raya Tiled + AVX2 (oracle/tiled.c), CPU baseline"})
        return rows

    path = kernel_bench.run(ROOT, None if args.no_cpu_baseline else cpu_rows)
    print(json.dumps({"raya_bench": path}), flush=True)


def main():
    args = parse()
    if args.raya_bench:
        raya_bench(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
