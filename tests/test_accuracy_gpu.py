"""Accuracy of the CUDA kernels beyond the reference's own test inputs, on a B200.

* Values with a non-zero mean over long key spans.  The reference's tests and
  goldens draw V with mean 0, which hides any error proportional to |O|.  The
  tensor core's accumulation in tensor memory truncates toward zero (about
  0.5 ulp of the accumulator per MMA): summing every key tile's PV product
  there put 1.6e-4 of absolute error into outputs near 1 on a Full mask at
  seq 8192.  These cases hold the kernels to the parity bar with V shifted to
  a mean of 1, against an fp64 dense softmax, and check that the signed error
  does not lean toward zero.
* Relative error at a floor of 1e-3 (the tests' own bar uses 1e-2, because
  next to zero relative error is noise): the default kernels on slices of the
  c2 and c5 configurations, next to the CPU Tiled restatement against the
  Naive one at the same floor.  The GPU may be at most twice as far from
  Naive as Tiled is, over the slices taken together (measured: 1.64x on c2,
  1.54x on c5; the inputs are fixed, so the figure does not move between
  runs).
"""
import numpy as np
import pytest

import oracle
import raya_b200 as rb
from raya_b200.workloads import CONFIGS
from _util import ATOL, cuda_device_run

pytestmark = pytest.mark.gpu

LONG_SPANS = [
    ("full-4096", oracle.Problem(1, 1, 4096, 64, mask=oracle.MASK_FULL)),
    ("block3-b128-4096", oracle.Problem(1, 2, 4096, 64, mask=oracle.MASK_BLOCK, block=128, halo=1)),
    ("block5-b256-4096", oracle.Problem(1, 2, 4096, 64, mask=oracle.MASK_BLOCK, block=256, halo=2)),
    ("window64-4096", oracle.Problem(1, 2, 4096, 64, mask=oracle.MASK_WINDOW, window=64)),
    ("block1-b256-2048", oracle.Problem(2, 2, 2048, 64, mask=oracle.MASK_BLOCK, block=256, halo=0)),
]


@pytest.mark.parametrize("kernel", [rb.KERNEL_AUTO, rb.KERNEL_TC32_WS, rb.KERNEL_TC32_WS2, rb.KERNEL_TC16_WS,
                                    rb.KERNEL_TC16_WS2, rb.KERNEL_TILED64])
@pytest.mark.parametrize("name,p", LONG_SPANS, ids=[n for n, _ in LONG_SPANS])
def test_values_with_nonzero_mean_over_long_spans(cuda_device, kernel, name, p):
    q, k, v = oracle.qkv(p.numel, 2024)
    v = (v + np.float32(1.0)).astype(np.float32)  # the reference tests' U(-1, 1) shifted to U(0, 2): outputs near 1
    valid = np.full(p.batch, p.seq, dtype=np.int32)
    valid[-1] = p.seq - 333  # a ragged tail
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel).astype(np.float64)
    want = oracle.dense_reference(p, q, k, v, valid)
    err = float(np.abs(got - want).max())
    assert err < ATOL, f"{name} kernel {kernel}: max abs {err:.3e} against fp64 (bar {ATOL:g})"
    # no systematic shrink toward zero: the signed error averages near 0
    rows = np.abs(want) > 0.5
    bias = float(np.mean((got - want)[rows] * np.sign(want[rows])))
    assert abs(bias) < 2e-6, f"{name} kernel {kernel}: mean signed error {bias:.3e}"


def _slice_inputs(w, bh):
    import torch

    n = w.seq * w.head_dim
    x = [torch.empty(n, device="cuda") for _ in range(3)]
    for t in range(3):
        rb.fill_normal(x[t], w.seed, t, bh * n, w.stddev)
    return x


@pytest.mark.parametrize("name,picks", [("c2", [0, 5, 77, 383]), ("c5", [0, 1000, 2047, 4095])])
def test_relative_error_at_the_1e3_floor(cuda_device, name, picks):
    import torch

    w = CONFIGS[name]
    valid = w.valid_len()
    worst = {"gpu": {1e-3: 0.0, 1e-2: 0.0}, "tiled": {1e-3: 0.0, 1e-2: 0.0}}
    for bh in picks:
        vl = [int(valid[bh // w.heads])]
        x = _slice_inputs(w, bh)
        shape = rb.AttnShape(heads=1, seq=w.seq, head_dim=w.head_dim, batch=1)
        params = rb.AttnParams.new(rb.Mask.block(w.halo), vl, w.head_dim, block=w.block)
        o = torch.empty_like(x[0])
        rb.Cuda().attend_device(shape, params, *x, o)
        rb.sync_status()
        p = oracle.Problem(1, 1, w.seq, w.head_dim, mask=oracle.MASK_BLOCK, block=w.block, halo=w.halo)
        hq, hk, hv = (t.cpu().numpy() for t in x)
        naive = oracle.naive(p, hq, hk, hv, vl).astype(np.float64)
        tiled = oracle.tiled(p, hq, hk, hv, vl).astype(np.float64)
        gpu = o.cpu().numpy().astype(np.float64)
        for floor in (1e-3, 1e-2):
            big = np.abs(naive) >= floor
            for key, arr in (("gpu", gpu), ("tiled", tiled)):
                rel = float((np.abs(arr - naive)[big] / np.abs(naive[big])).max())
                worst[key][floor] = max(worst[key][floor], rel)
    print(f"{name}: max rel vs Naive, floor 1e-3: GPU {worst['gpu'][1e-3]:.3e}, Tiled {worst['tiled'][1e-3]:.3e}; "
          f"floor 1e-2: GPU {worst['gpu'][1e-2]:.3e}, Tiled {worst['tiled'][1e-2]:.3e}")
    assert worst["gpu"][1e-3] <= 2.0 * worst["tiled"][1e-3]
    assert worst["gpu"][1e-2] < 1e-4


SCALES = [(1.0, 1.0, 1.0), (1e3, 1e-3, 1e5), (1e-4, 1e4, 1e-6), (3e4, 1e-4, 7e4), (2.0 ** -20, 2.0 ** 20, 2.0 ** 30)]


@pytest.mark.parametrize("kernel", [rb.KERNEL_AUTO, rb.KERNEL_TC32_WS, rb.KERNEL_TC32_WS2, rb.KERNEL_TC16_WS,
                                    rb.KERNEL_TC16_WS2])
@pytest.mark.parametrize("sq,sk,sv", SCALES, ids=[f"q{a:g}-k{b:g}-v{c:g}" for a, b, c in SCALES])
def test_operand_magnitudes(cuda_device, kernel, sq, sk, sv):
    """q, k and v far from unit size, past fp16's range (65504) and below its
    normal range (6.1e-5): the 3xFP16 kernel scales each q row and each
    64-key K and V tile by a power of two, the 3xTF32 kernel needs none.  The
    scores are the same as at unit size (sq * sk = 1 for all but the last
    case), so the error is measured relative to the scale of V."""
    p = oracle.Problem(2, 2, 700, 64, mask=oracle.MASK_BLOCK, block=128, halo=1)
    q, k, v = oracle.qkv(p.numel, 77)
    q, k, v = ((x.astype(np.float64) * s).astype(np.float32) for x, s in ((q, sq), (k, sk), (v, sv)))
    valid = [700, 411]
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel).astype(np.float64)
    want = oracle.dense_reference(p, q, k, v, np.array(valid, dtype=np.int32))
    err = float(np.abs(got - want).max()) / sv
    assert err < ATOL, f"kernel {kernel}, scales ({sq:g}, {sk:g}, {sv:g}): max abs / |v| {err:.3e}"


@pytest.mark.parametrize("kernel", [rb.KERNEL_TC32_WS2, rb.KERNEL_TC16_WS, rb.KERNEL_TC16_WS2])
def test_magnitudes_varying_by_key_tile(cuda_device, kernel):
    """Operand sizes that change by 2^20 to 2^40 from one 64-key tile to the
    next (so every K and V tile of the 3xFP16 kernel gets its own scale, V
    tiles beyond fp16's range) and q rows whose size falls by 2^20 along the
    sequence.  The scores stay O(1), so fp32 arithmetic gives ~1e-7 of the
    largest |V|; the outputs must match fp64 to the parity bar on that scale."""
    p = oracle.Problem(1, 2, 640, 64, mask=oracle.MASK_FULL)
    q, k, v = oracle.qkv(p.numel, 91)
    pos = np.arange(p.seq)
    even = (pos // 64) % 2 == 0
    row_scale = 2.0 ** (-20.0 * pos / p.seq)          # per query row: 1 .. 2^-20
    k_scale = np.where(even, 1.0, 2.0 ** -20)          # per key tile
    v_scale = np.where(even, 2.0 ** 20, 2.0 ** -20)    # per key tile
    shape = (p.batch, p.heads, p.seq, p.head_dim)
    q = (q.reshape(shape) * row_scale[None, None, :, None]).astype(np.float32).ravel()
    k = (k.reshape(shape) * k_scale[None, None, :, None]).astype(np.float32).ravel()
    v = (v.reshape(shape) * v_scale[None, None, :, None]).astype(np.float32).ravel()
    got = cuda_device_run(p, q, k, v, kernel=kernel).astype(np.float64)
    want = oracle.dense_reference(p, q, k, v, np.full(p.batch, p.seq, dtype=np.int32))
    # each output row is a convex combination of V rows: its error scale is max |V|
    vmax = float(np.abs(v).max())
    err = float(np.abs(got - want).max()) / vmax
    assert err < ATOL, f"kernel {kernel}: max abs / max|v| {err:.3e}"
