"""CPU oracle for raya's block-local attention: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs import this package, and only as the checker or the timed CPU
baseline.  The product (``raya_b200``) never imports it.

Contents:
  * ``naive`` / ``naive_range``: ctypes over ``_build/liboracle.so``, the C
    restatement of ``Naive::attend`` (crates/raya-kernels/src/naive.rs:13-65).
  * ``tiled``: the C restatement of ``Tiled`` + AVX2 micro-kernels
    (crates/raya-kernels/src/tiled/tile.rs:27-151, simd/avx2.rs:23-74).
  * ``dense_reference``: numpy fp64 dense masked softmax, the independent
    check of crates/raya-kernels/tests/common/mod.rs:39-84.
  * ``rand_vec`` / ``lcg_fill``: the reference tests' input generators
    (tests/common/mod.rs:6-18, tests/masks_edges.rs:6-14).
  * ``build()``: compiles the C sources with the committed Makefile.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

MASK_BLOCK, MASK_WINDOW, MASK_FULL = 0, 1, 2


class _Desc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seq", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("block", ctypes.c_int64),
        ("mask", ctypes.c_int32),
        ("halo", ctypes.c_int32),
        ("window", ctypes.c_int64),
        ("scale", ctypes.c_float),
    ]


@dataclass(frozen=True)
class Problem:
    """One attention call: ``[batch][heads][seq][head_dim]`` fp32 tensors."""

    batch: int
    heads: int
    seq: int
    head_dim: int
    mask: int = MASK_BLOCK
    block: int = 128
    halo: int = 1
    window: int = 64
    scale: float | None = None

    def desc(self) -> _Desc:
        scale = self.scale
        if scale is None:
            # attention.rs:103: 1.0 / (head_dim as f32).sqrt(), in f32
            scale = float(np.float32(1.0) / np.sqrt(np.float32(self.head_dim)))
        return _Desc(self.batch, self.heads, self.seq, self.head_dim, self.block,
                     self.mask, self.halo, self.window, scale)

    @property
    def numel(self) -> int:
        return self.batch * self.heads * self.seq * self.head_dim


def build(quiet: bool = True) -> str:
    """Compile the oracle with its Makefile; returns the library path."""
    out = subprocess.run(["make", "-C", _HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{out.stdout}\n{out.stderr}")
    if not quiet:
        print(out.stdout)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        ip = ctypes.POINTER(ctypes.c_int32)
        dp = ctypes.POINTER(_Desc)
        L.oracle_naive_range.argtypes = [dp, fp, fp, fp, fp, ip, ctypes.c_int64, ctypes.c_int64]
        L.oracle_naive_range.restype = None
        L.oracle_tiled.argtypes = [dp, fp, fp, fp, fp, ip, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int, ctypes.c_int]
        L.oracle_tiled.restype = ctypes.c_int
        L.oracle_count.argtypes = [dp, ip, ctypes.POINTER(ctypes.c_uint64),
                                   ctypes.POINTER(ctypes.c_uint64)]
        L.oracle_key_range.argtypes = [dp, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.POINTER(ctypes.c_int64),
                                       ctypes.POINTER(ctypes.c_int64)]
        L.oracle_rand_vec.argtypes = [fp, ctypes.c_size_t, ctypes.c_uint64]
        L.oracle_lcg_fill.argtypes = [fp, ctypes.c_size_t, ctypes.c_uint32]
        L.oracle_cpu_has_avx2_fma.restype = ctypes.c_int
        i64 = ctypes.c_int64
        L.oracle_split_qkv.argtypes = [fp, i64, i64, i64, fp, fp, fp]
        L.oracle_rope_inplace.argtypes = [fp, i64, i64, i64, ctypes.c_float]
        L.oracle_merge_ctx.argtypes = [fp, i64, i64, i64, fp]
        _lib = L
    return _lib


def _f32(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _valid_ptr(valid_len):
    if valid_len is None:
        return None, None
    arr = np.ascontiguousarray(np.asarray(valid_len, dtype=np.int32))
    return arr, arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def naive(p: Problem, q, k, v, valid_len=None, bh_range=None) -> np.ndarray:
    """Naive::attend restated (naive.rs:13-65); returns ``out``.

    ``bh_range=(bh0, bh1)`` computes only those flattened (batch*heads)
    slices; other slices of the result are left zero."""
    out = np.zeros(p.numel, dtype=np.float32)
    keep, vp = _valid_ptr(valid_len)
    bh0, bh1 = bh_range if bh_range is not None else (0, p.batch * p.heads)
    d = p.desc()
    lib().oracle_naive_range(ctypes.byref(d), _f32(q), _f32(k), _f32(v), _f32(out), vp,
                             bh0, bh1)
    del keep
    return out


def tiled(p: Problem, q, k, v, valid_len=None, threads: int = 1, backend: int = 1,
          bh_range=None, out: np.ndarray | None = None) -> np.ndarray:
    """Tiled::attend restated (tile.rs + avx2.rs), ``threads`` workers."""
    if out is None:
        out = np.zeros(p.numel, dtype=np.float32)
    keep, vp = _valid_ptr(valid_len)
    bh0, bh1 = bh_range if bh_range is not None else (0, p.batch * p.heads)
    d = p.desc()
    lib().oracle_tiled(ctypes.byref(d), _f32(q), _f32(k), _f32(v), _f32(out), vp,
                       bh0, bh1, threads, backend)
    del keep
    return out


def count(p: Problem, valid_len=None) -> tuple[int, int]:
    """(allowed pairs, valid query rows) over batch and heads."""
    keep, vp = _valid_ptr(valid_len)
    pairs, rows = ctypes.c_uint64(), ctypes.c_uint64()
    d = p.desc()
    lib().oracle_count(ctypes.byref(d), vp, ctypes.byref(pairs), ctypes.byref(rows))
    del keep
    return pairs.value, rows.value


def key_range(p: Problem, i: int, valid: int) -> tuple[int, int]:
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    d = p.desc()
    lib().oracle_key_range(ctypes.byref(d), i, valid, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def cpu_has_avx2_fma() -> bool:
    return bool(lib().oracle_cpu_has_avx2_fma())


def rand_vec(n: int, seed: int) -> np.ndarray:
    """tests/common/mod.rs:6-18 (xorshift, uniform [-1, 1])."""
    out = np.empty(n, dtype=np.float32)
    lib().oracle_rand_vec(_f32(out), n, seed)
    return out


def qkv(numel: int, seed: int):
    """tests/common/mod.rs:20-27: q, k, v from seeds seed, seed+1, seed+2."""
    return rand_vec(numel, seed), rand_vec(numel, seed + 1), rand_vec(numel, seed + 2)


def lcg_fill(n: int, seed: int) -> np.ndarray:
    """tests/masks_edges.rs:6-14 (LCG, [-0.5, 0.5))."""
    out = np.empty(n, dtype=np.float32)
    lib().oracle_lcg_fill(_f32(out), n, seed)
    return out


def allowed_matrix(p: Problem, valid: int) -> np.ndarray:
    """Boolean [seq, seq]: query i may attend key j (mask and valid_len)."""
    L = p.seq
    i = np.arange(L)[:, None]
    j = np.arange(L)[None, :]
    if p.mask == MASK_BLOCK:
        m = np.abs(i // p.block - j // p.block) <= p.halo
    elif p.mask == MASK_WINDOW:
        m = np.abs(i - j) <= p.window
    else:
        m = np.ones((L, L), dtype=bool)
    return m & (i < valid) & (j < valid)


def dense_reference(p: Problem, q, k, v, valid_len=None) -> np.ndarray:
    """Independent fp64 dense masked softmax (tests/common/mod.rs:39-84):
    full [seq, seq] scores, boolean mask, zero rows where nothing is allowed.
    Only for small problems."""
    L, D = p.seq, p.head_dim
    scale = float(p.desc().scale)
    q4 = np.asarray(q, dtype=np.float64).reshape(p.batch, p.heads, L, D)
    k4 = np.asarray(k, dtype=np.float64).reshape(p.batch, p.heads, L, D)
    v4 = np.asarray(v, dtype=np.float64).reshape(p.batch, p.heads, L, D)
    out = np.zeros((p.batch, p.heads, L, D), dtype=np.float64)
    for b in range(p.batch):
        valid = L if valid_len is None else int(valid_len[b])
        allow = allowed_matrix(p, valid)
        any_row = allow.any(axis=1)
        for h in range(p.heads):
            s = (q4[b, h] @ k4[b, h].T) * scale
            s = np.where(allow, s, -np.inf)
            mx = np.where(any_row, s.max(axis=1), 0.0)
            e = np.where(allow, np.exp(s - mx[:, None]), 0.0)
            tot = e.sum(axis=1)
            w = np.divide(e, tot[:, None], out=np.zeros_like(e), where=tot[:, None] > 0)
            out[b, h] = w @ v4[b, h]
    return out.reshape(-1)


def encoder_attend(qkv: np.ndarray, batch: int, seq: int, heads: int, head_dim: int, mask: int,
                   block: int, halo: int, window: int, valid_len, rope_theta: float | None) -> np.ndarray:
    """The caller's whole attention step, restated: per batch entry,
    split_qkv (encoder.rs:34-53), rope on q and k (ops.rs:110-141) when
    rope_theta is given, Naive attention, and the context back to
    [seq][heads*head_dim] (encoder.rs:82-90).  Returns ctx
    [batch][seq][heads*head_dim]."""
    L = lib()
    n = seq * heads * head_dim
    ctx = np.zeros(batch * n, dtype=np.float32)
    p = Problem(1, heads, seq, head_dim, mask=mask, block=block, halo=halo, window=window)
    for b in range(batch):
        src = np.ascontiguousarray(qkv[b * 3 * n:(b + 1) * 3 * n])
        q, k, v = (np.empty(n, dtype=np.float32) for _ in range(3))
        L.oracle_split_qkv(_f32(src), seq, heads, head_dim, _f32(q), _f32(k), _f32(v))
        if rope_theta:
            L.oracle_rope_inplace(_f32(q), heads, seq, head_dim, rope_theta)
            L.oracle_rope_inplace(_f32(k), heads, seq, head_dim, rope_theta)
        out = naive(p, q, k, v, [int(np.broadcast_to(valid_len, (batch,))[b])])
        part = np.empty(n, dtype=np.float32)
        L.oracle_merge_ctx(_f32(out), seq, heads, head_dim, _f32(part))
        ctx[b * n:(b + 1) * n] = part
    return ctx
