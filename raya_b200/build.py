"""Builds libraya_attn.so in-tree (raya_b200/_lib/) with nvcc for sm_100a.

    python raya_b200/build.py          # build if sources are newer
    python raya_b200/build.py --force  # rebuild
    python raya_b200/build.py --ptxas  # also print -Xptxas -v resource usage

It is run as a script (or loaded by file path from __graft_entry__.build()):
importing the raya_b200 package loads the library, which may not exist yet.

The library is a plain shared object with a C ABI (include/raya_attn.h); the
CUDA runtime is linked statically, so it loads next to torch's own runtime.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "libraya_attn.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-O2,-Wall", "-shared", "-cudart", "static"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(ROOT, "include", "raya_attn.h"), os.path.abspath(__file__)]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in deps())


def build(force: bool = False, ptxas: bool = False, quiet: bool = True) -> str:
    if not force and not ptxas and not stale():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-o", LIB, *sources()]
    if ptxas:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{res.stdout}\n{res.stderr}")
    if ptxas or not quiet:
        sys.stdout.write(res.stdout + res.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, ptxas=args.ptxas, quiet=False))
