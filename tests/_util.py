"""Shared helpers of the parity tests (CUDA path vs the CPU oracle)."""
from __future__ import annotations

import numpy as np

import oracle
import raya_b200 as rb

# Parity bar: max-abs 1e-5 over all elements (the reference's own bar,
# goldens.rs:15, equivalence.rs:26) and max-rel 1e-4 over elements whose
# reference magnitude is at least 1e-2.  Relative error is ill-posed next to
# zero: outputs are convex combinations of O(1) values, so fp32 rounding
# leaves ~1e-7 absolute error everywhere.  The golden's own two tensors
# (Laya's native reference and its PyTorch kernel) differ by 1.1e-4 relative
# over |ref| >= 1e-3 but by 1.5e-5 over |ref| >= 1e-2 (92% of elements).
ATOL = 1e-5
RTOL = 1e-4
REL_FLOOR = 1e-2


def mask_of(p: oracle.Problem) -> rb.Mask:
    if p.mask == oracle.MASK_BLOCK:
        return rb.Mask.block(p.halo)
    if p.mask == oracle.MASK_WINDOW:
        return rb.Mask.sliding(p.window)
    return rb.Mask.FULL


def shape_params(p: oracle.Problem, valid=None):
    shape = rb.AttnShape(heads=p.heads, seq=p.seq, head_dim=p.head_dim, batch=p.batch)
    vl = p.seq if valid is None else valid
    params = rb.AttnParams.new(mask_of(p), vl, p.head_dim, block=p.block)
    if p.scale is not None:
        params = rb.AttnParams(mask=params.mask, block=params.block, valid_len=vl, scale=p.scale)
    return shape, params


def cuda_device_run(p: oracle.Problem, q, k, v, valid=None, kernel=rb.KERNEL_AUTO, fill=7.0):
    """Runs the CUDA kernel on device copies; returns the output as numpy."""
    import torch

    shape, params = shape_params(p, valid)
    dev = torch.device("cuda", 0)
    tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (q, k, v))
    out = torch.full((p.numel,), fill, dtype=torch.float32, device=dev)
    vl = torch.from_numpy(params.valid_array(p.batch)).to(dev)
    rb.Cuda().attend_device(shape, params, tq, tk, tv, out, valid_len=vl, kernel=kernel)
    rb.sync_status()
    return out.cpu().numpy()


def cuda_host_run(p: oracle.Problem, q, k, v, valid=None, fill=7.0):
    """The drop-in host-buffer call (AttentionKernel::attend)."""
    shape, params = shape_params(p, valid)
    out = np.full(p.numel, fill, dtype=np.float32)
    rb.Cuda().attend(shape, params, q, k, v, out)
    return out


def assert_close(got, want, what="", atol=ATOL, rtol=RTOL):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, what
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    diff = np.abs(got - want)
    amax = float(diff.max()) if diff.size else 0.0
    big = np.abs(want) >= REL_FLOOR
    rmax = float((diff[big] / np.abs(want[big])).max()) if big.any() else 0.0
    assert amax < atol, f"{what}: max abs diff {amax:.3e} (rel {rmax:.3e})"
    assert rmax < rtol, f"{what}: max rel diff {rmax:.3e} (abs {amax:.3e})"
    return amax, rmax


def padded_rows_exact_zero(out, p: oracle.Problem, valid):
    o = np.asarray(out).reshape(p.batch, p.heads, p.seq, p.head_dim)
    for b in range(p.batch):
        vb = p.seq if valid is None else int(np.broadcast_to(valid, (p.batch,))[b])
        tail = o[b, :, vb:, :]
        if tail.size:
            assert (tail == 0.0).all(), f"batch {b}: padded rows are not exactly zero"
            assert not np.signbit(tail).any(), f"batch {b}: padded rows hold -0.0"


def load_golden():
    import json
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "block_local_L256_h3.npz"))
    meta = json.loads(str(z["meta"]))
    return meta, {n: z[n] for n in ("q", "k", "v", "reference", "kernel")}
