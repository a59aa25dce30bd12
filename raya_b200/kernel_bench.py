"""raya's kernel-bench result file, produced by the B200 kernel.

raya's `cargo bench -p raya-kernels --bench local_attention`
(crates/raya-kernels/benches/local_attention.rs:72-173) times one layer of
block-local attention (16 heads, head_dim 64, block 128, masks Block3 and
Window64, seq from RAYA_BENCH_SEQS, default 2048,4096,8192; inputs uniform
[-1, 1]) and writes results/kernel-bench/<timestamp>.json in the contract of
specs/007-block-local-kernel/contracts/bench-output.md:8-24.  `run()` does the
same on the GPU and writes the same document, with the GPU described in the
metadata, so the two result sets can be read side by side.
"""
from __future__ import annotations

import json
import os
import statistics
import subprocess
import time

import numpy as np

HEADS = 16
HEAD_DIM = 64
SAMPLES = 10

# meta.rs:5-10 — the label never claims more than the caller says.
LABELS = {"1": "target machine", "cloud-agent": "cloud-agent hardware, indicative only"}
UNLABELED = "unlabeled machine, indicative only"


def seqs() -> list[int]:
    """benches/local_attention.rs:35-41."""
    raw = os.environ.get("RAYA_BENCH_SEQS", "")
    out = [int(x) for x in raw.split(",") if x.strip().isdigit()]
    return out or [2048, 4096, 8192]


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return ""


def _git_commit(root: str) -> str:
    try:
        return subprocess.run(["git", "-C", root, "rev-parse", "--short", "HEAD"], capture_output=True,
                              text=True, timeout=10).stdout.strip()
    except (OSError, subprocess.SubprocessError):
        return ""


def metadata(root: str, threads: int) -> dict:
    """BenchMetadata (meta.rs:12-103) plus the GPU that ran."""
    import torch

    props = torch.cuda.get_device_properties(0)
    try:
        nvcc = subprocess.run(["nvcc", "--version"], capture_output=True, text=True, timeout=10).stdout
        nvcc = nvcc.strip().splitlines()[-1]
    except (OSError, subprocess.SubprocessError):
        nvcc = ""
    try:
        smi = subprocess.run(["nvidia-smi", "--query-gpu=driver_version,clocks.max.sm", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=10).stdout.strip().splitlines()[0]
        driver, max_sm = (x.strip() for x in smi.split(","))
    except (OSError, subprocess.SubprocessError, IndexError, ValueError):
        driver, max_sm = "", ""
    return {
        "label": LABELS.get(os.environ.get("RAYA_TARGET_MACHINE", ""), UNLABELED),
        "cpu_model": _cpu_model(), "logical_cpus": os.cpu_count() or 0,
        "physical_cpus": len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else 0,
        "threads": threads, "features": ["tcgen05-3xtf32", "tiled64", "ffma2", "tma"], "backend": "sm_100a",
        "rustflags": "", "rustc": "", "git_commit": _git_commit(root),
        "timestamp": f"unix:{int(time.time())}",
        "gpu": props.name, "gpu_sms": props.multi_processor_count, "gpu_max_sm_clock": max_sm,
        "driver": driver, "nvcc": nvcc, "n_gpus": 1,
    }


def _time_calls(fn, samples: int, warmup: int = 3) -> tuple[float, float]:
    """Mean and standard deviation in ms of `samples` calls, each timed on
    the device with its own CUDA events."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(samples):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.mean(times), statistics.stdev(times) if len(times) > 1 else 0.0


def run(root: str, cpu_rows=None) -> str:
    """Times the GPU kernel on every (seq, mask) of the reference bench and
    writes the result file.  `cpu_rows(seq, mask) -> list[dict]` may add rows
    measured on the host (the bench's CPU baseline); returns the file path."""
    import torch

    import raya_b200 as rb

    dev = torch.device("cuda", 0)
    kern = rb.Cuda()
    results = []
    for seq in seqs():
        shape = rb.AttnShape(heads=HEADS, seq=seq, head_dim=HEAD_DIM)
        g = torch.Generator(device=dev).manual_seed(42)  # local_attention.rs:95 uses seed 42
        q, k, v = (torch.rand(shape.numel(), generator=g, device=dev) * 2 - 1 for _ in range(3))
        out = torch.empty_like(q)
        for mask, name in ((rb.Mask.BLOCK3, "block3"), (rb.Mask.WINDOW64, "window64")):
            params = rb.AttnParams.new(mask, seq, HEAD_DIM)
            dvalid = torch.tensor([seq], dtype=torch.int32, device=dev)
            mean, sd = _time_calls(lambda: kern.attend_device(shape, params, q, k, v, out, valid_len=dvalid),
                                   SAMPLES)
            st = rb.stage_times(shape, params, q, k, v, out, valid_len=dvalid, kernel=rb.KERNEL_AUTO)
            pairs, _ = rb.work(shape, params)
            results.append({
                "kernel": "cuda-b200", "mask": name, "backend": "sm_100a", "seq": seq, "heads": HEADS,
                "head_dim": HEAD_DIM, "threads": 1, "mean_ms": mean, "stddev_ms": sd, "samples": SAMPLES,
                "stages": {"qk_pct": st.get("qk_pct", 0.0), "softmax_pct": st.get("softmax_pct", 0.0),
                           "pv_pct": st.get("pv_pct", 0.0)},
                "gflops": 4 * HEAD_DIM * pairs / (mean * 1e-3) / 1e9,
            })
            if cpu_rows is not None:
                results.extend(cpu_rows(seq, name, q, k, v))
        del q, k, v, out
    meta = metadata(root, threads=1)
    doc = {"label": meta["label"], "metadata": meta, "results": results}
    out_dir = os.path.join(root, "results", "kernel-bench")
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, meta["timestamp"].replace(":", "-") + ".json")
    with open(path, "w") as f:
        json.dump(doc, f, indent=2)
    return path
