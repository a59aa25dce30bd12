"""CUDA path vs the CPU oracle, on a B200.

Cases follow the reference's kernel tests (crates/raya-kernels/tests/):
equivalence.rs (edge lengths, padded tails, head counts and dims), masking.rs
(mask exactness, exact-zero padding, extreme logits), goldens.rs (Laya's
block_local golden), masks_edges.rs (single valid row, nothing valid) — run
through both CUDA kernels and the host-buffer drop-in call — plus the
extensions this path adds: block sizes other than 128, halo 0/1/2, batch > 1
with ragged valid lengths, windows, Full.
"""
import numpy as np
import pytest

import oracle
import raya_b200 as rb
from _util import (assert_close, cuda_device_run, cuda_host_run, load_golden,
                   padded_rows_exact_zero)

pytestmark = pytest.mark.gpu

KERNELS_D64 = [rb.KERNEL_TILED64, rb.KERNEL_ROWWISE, rb._lib.KERNEL_TC32_WS, rb._lib.KERNEL_TC32_WS2,
               rb._lib.KERNEL_TC16_WS, rb._lib.KERNEL_TC16_WS2]
# every compiled variant of the tiled kernel (warps per CTA x K/V stages)
TILED_VARIANTS = [rb.KERNEL_TILED64] + sorted(rb._lib.KERNEL_TILED64_VARIANTS.values())
# every head_dim-64 kernel: the FFMA variants, rowwise, and the 3xTF32 tensor-core kernels
ALL_D64 = TILED_VARIANTS + [rb.KERNEL_ROWWISE, rb._lib.KERNEL_TC32_WS, rb._lib.KERNEL_TC32_WS2,
                            rb._lib.KERNEL_TC16_WS, rb._lib.KERNEL_TC16_WS2]
B3 = dict(mask=oracle.MASK_BLOCK, block=128, halo=1)
W64 = dict(mask=oracle.MASK_WINDOW, window=64)


def _qkv(p, seed):
    return oracle.qkv(p.numel, seed)


@pytest.mark.parametrize("kernel", KERNELS_D64)
def test_block_local_golden(cuda_device, kernel):
    """goldens.rs:35-80: Laya's block_local golden, [16, 256, 64], block 128."""
    meta, g = load_golden()
    assert meta["pattern"] == "block_local" and meta["block"] == 128
    h = len(meta["heads_kept"])
    p = oracle.Problem(1, h, meta["length"], meta["head_dim"], **B3)
    q, k, v = (np.ascontiguousarray(g[n].reshape(-1)) for n in ("q", "k", "v"))
    got = cuda_device_run(p, q, k, v, kernel=kernel)
    for name in ("reference", "kernel"):
        assert_close(got, g[name].reshape(-1), f"golden `{name}`", atol=meta["tolerance"])
    assert_close(got, oracle.naive(p, q, k, v), "oracle")


def test_block_local_golden_host_call(cuda_device):
    meta, g = load_golden()
    p = oracle.Problem(1, len(meta["heads_kept"]), 256, 64, **B3)
    q, k, v = (np.ascontiguousarray(g[n].reshape(-1)) for n in ("q", "k", "v"))
    got = cuda_host_run(p, q, k, v)
    assert_close(got, g["reference"].reshape(-1), "golden via host call", atol=meta["tolerance"])


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
@pytest.mark.parametrize("seq", [1, 127, 128, 129, 1000, 2048])
@pytest.mark.parametrize("kernel", ALL_D64)
def test_matches_oracle_at_edge_lengths(cuda_device, mask, seq, kernel):
    """equivalence.rs:29-42."""
    heads = 2 if seq >= 1000 else 3
    p = oracle.Problem(1, heads, seq, 64, **mask)
    q, k, v = _qkv(p, 100 + seq)
    got = cuda_device_run(p, q, k, v, kernel=kernel)
    assert_close(got, oracle.naive(p, q, k, v), f"seq {seq}")


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
@pytest.mark.parametrize("seq,valid", [(300, 263), (1000, 963), (256, 1), (256, 0), (129, 128)])
@pytest.mark.parametrize("kernel", KERNELS_D64)
def test_matches_oracle_with_padded_tail(cuda_device, mask, seq, valid, kernel):
    """equivalence.rs:44-66."""
    p = oracle.Problem(1, 2, seq, 64, **mask)
    q, k, v = _qkv(p, 100 + seq)
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel)
    assert_close(got, oracle.naive(p, q, k, v, [valid]), f"seq {seq} valid {valid}")
    padded_rows_exact_zero(got, p, [valid])


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
@pytest.mark.parametrize("heads,seq,d", [(16, 512, 64), (2, 300, 8), (2, 300, 40), (2, 300, 96),
                                         (2, 300, 16), (2, 300, 256)])
def test_matches_oracle_heads_and_head_dims(cuda_device, mask, heads, seq, d):
    """equivalence.rs:68-112 (head_dim != 64 runs the rowwise kernel)."""
    p = oracle.Problem(1, heads, seq, d, **mask)
    q, k, v = _qkv(p, 100 + seq)
    got = cuda_device_run(p, q, k, v)
    assert_close(got, oracle.naive(p, q, k, v), f"h{heads} d{d}")


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
@pytest.mark.parametrize("d", [8, 64])
def test_masks_are_exact(cuda_device, mask, d):
    """masking.rs:20-61: one-hot V row of key j; weight > 0 iff allowed, == 0.0 otherwise."""
    n = 300
    p = oracle.Problem(1, 1, n, d, **mask)
    q, k = oracle.rand_vec(p.numel, 5), oracle.rand_vec(p.numel, 6)
    m = rb.Mask.BLOCK3 if mask is B3 else rb.Mask.WINDOW64
    kernels = [rb.KERNEL_AUTO] + ([rb.KERNEL_ROWWISE, rb._lib.KERNEL_TC32_WS, rb._lib.KERNEL_TC32_WS2,
                                   rb._lib.KERNEL_TC16_WS, rb._lib.KERNEL_TC16_WS2] if d == 64 else [])
    for kernel in kernels:
        for j in [0, 1, 63, 64, 65, 127, 128, 129, 191, 255, 256, 299]:
            v = np.zeros(p.numel, dtype=np.float32)
            v[j * d] = 1.0
            out = cuda_device_run(p, q, k, v, kernel=kernel).reshape(n, d)
            w = out[:, 0]
            for i in range(n):
                if m.allows(i, j):
                    assert w[i] > 0.0, f"kernel {kernel}: query {i} should see key {j}"
                else:
                    assert w[i] == 0.0, f"kernel {kernel}: query {i} must not see key {j}"


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
@pytest.mark.parametrize("d", [16, 64])
def test_padding_and_empty_rows_are_exact_zeros(cuda_device, mask, d):
    """masking.rs:63-91."""
    p = oracle.Problem(1, 2, 200, d, **mask)
    q, k, v = oracle.qkv(p.numel, 9)
    for valid in (0, 1, 150):
        for run in (lambda: cuda_device_run(p, q, k, v, valid=valid, fill=1.0),
                    lambda: cuda_host_run(p, q, k, v, valid=valid, fill=1.0)):
            out = run()
            padded_rows_exact_zero(out, p, [valid])
            assert np.isfinite(out).all()
            assert_close(out, oracle.naive(p, q, k, v, [valid]), f"valid {valid}")


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
@pytest.mark.parametrize("kernel", KERNELS_D64)
def test_extreme_logits_are_stable_and_match_the_oracle(cuda_device, mask, kernel):
    """masking.rs:93-126: q and k scaled by 400 (logits ~ 1e4)."""
    p = oracle.Problem(1, 2, 300, 64, **mask)
    q, k, v = oracle.qkv(p.numel, 21)
    q, k = q * np.float32(400.0), k * np.float32(400.0)
    want = oracle.naive(p, q, k, v)
    assert np.isfinite(want).all()
    got = cuda_device_run(p, q, k, v, kernel=kernel)
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() < 1e-5


def test_a_single_valid_row_attends_only_to_itself(cuda_device):
    """masks_edges.rs:90-107 (Full and Sliding(2), one valid row)."""
    for mask in (dict(mask=oracle.MASK_FULL), dict(mask=oracle.MASK_WINDOW, window=2)):
        p = oracle.Problem(1, 1, 5, 8, **mask)
        q, k, v = (oracle.lcg_fill(40, s) for s in (31, 32, 33))
        out = cuda_device_run(p, q, k, v, valid=1)
        assert np.abs(out[:8] - v[:8]).max() < 1e-6
        assert (out[8:] == 0.0).all()


def test_nothing_valid_gives_all_zero_rows(cuda_device):
    """masks_edges.rs:74-88."""
    p0 = oracle.Problem(1, 2, 7, 8)
    x = oracle.lcg_fill(p0.numel, 21)
    for mask in (dict(mask=oracle.MASK_FULL), dict(mask=oracle.MASK_WINDOW, window=4),
                 dict(mask=oracle.MASK_WINDOW, window=0), B3):
        p = oracle.Problem(1, 2, 7, 8, **mask)
        out = cuda_device_run(p, x, x, x, valid=0, fill=1.0)
        assert (out == 0.0).all()


@pytest.mark.parametrize("block", [32, 64, 128, 256, 48, 7, 1])
@pytest.mark.parametrize("halo", [0, 1, 2])
@pytest.mark.parametrize("kernel", ALL_D64)
def test_block_sizes_halos_and_ragged_batches(cuda_device, block, halo, kernel):
    """Extensions: any block size, halo, batch > 1 with per-sequence valid_len."""
    p = oracle.Problem(3, 2, 700, 64, mask=oracle.MASK_BLOCK, block=block, halo=halo)
    q, k, v = oracle.qkv(p.numel, 1000 + block + halo)
    valid = [700, 433, 64]
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel)
    assert_close(got, oracle.naive(p, q, k, v, valid), f"block {block} halo {halo}")
    padded_rows_exact_zero(got, p, valid)


@pytest.mark.parametrize("window", [0, 1, 31, 64, 100, 500])
@pytest.mark.parametrize("kernel", ALL_D64)
def test_windows_and_ragged_batches(cuda_device, window, kernel):
    p = oracle.Problem(2, 2, 520, 64, mask=oracle.MASK_WINDOW, window=window)
    q, k, v = oracle.qkv(p.numel, 2000 + window)
    valid = [520, 301]
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel)
    assert_close(got, oracle.naive(p, q, k, v, valid), f"window {window}")


@pytest.mark.parametrize("kernel", KERNELS_D64)
def test_full_mask_matches_dense_softmax(cuda_device, kernel):
    """masks_dense.rs / masks_edges.rs:65-72 (Full), with ragged batches."""
    p = oracle.Problem(2, 2, 300, 64, mask=oracle.MASK_FULL)
    q, k, v = (oracle.lcg_fill(p.numel, s) for s in (11, 12, 13))
    valid = [300, 150]
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel)
    assert_close(got, oracle.naive(p, q, k, v, valid), "full")
    assert np.abs(got - oracle.dense_reference(p, q, k, v, valid)).max() < 1e-5


def test_results_are_bitwise_reproducible_and_shard_invariant(cuda_device):
    """equivalence.rs:114-129 analogue: the result does not depend on how the
    work is split.  Two runs agree bit for bit, and computing the batch in two
    halves (as two GPU shards would) gives the same bits as one call."""
    p = oracle.Problem(4, 3, 700, 64, **B3)
    q, k, v = oracle.qkv(p.numel, 77)
    valid = [650, 700, 129, 1]
    one = cuda_device_run(p, q, k, v, valid=valid)
    two = cuda_device_run(p, q, k, v, valid=valid)
    assert np.array_equal(one, two)
    half = p.numel // 2
    ph = oracle.Problem(2, 3, 700, 64, **B3)
    a = cuda_device_run(ph, q[:half], k[:half], v[:half], valid=valid[:2])
    b = cuda_device_run(ph, q[half:], k[half:], v[half:], valid=valid[2:])
    assert np.array_equal(np.concatenate([a, b]), one)


@pytest.mark.parametrize("mask", [dict(mask=oracle.MASK_BLOCK, block=64, halo=1), W64,
                                  dict(mask=oracle.MASK_FULL)], ids=["block64", "window64", "full"])
@pytest.mark.parametrize("kernel", ALL_D64)
def test_padding_values_never_reach_the_output(cuda_device, mask, kernel):
    """Rows at or past valid_len are padding: the reference never reads them
    (naive.rs:37, tile.rs:80-87).  Filled with NaN and Inf here, they must not
    change a single valid output."""
    p = oracle.Problem(3, 2, 300, 64, **mask)
    q, k, v = oracle.qkv(p.numel, 31)
    valid = [263, 300, 7]
    q4, k4, v4 = (x.reshape(3, 2, 300, 64) for x in (q, k, v))
    for b, vl in enumerate(valid):
        q4[b, :, vl:] = np.nan
        k4[b, :, vl:] = np.inf
        v4[b, :, vl:] = np.nan
    want = oracle.naive(p, q, k, v, valid)
    assert np.isfinite(want).all()
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel)
    assert np.isfinite(got).all()
    assert_close(got, want, "NaN/Inf padding")
    padded_rows_exact_zero(got, p, valid)


@pytest.mark.parametrize("mask", [dict(mask=oracle.MASK_BLOCK, block=64, halo=1), B3, W64,
                                  dict(mask=oracle.MASK_FULL)], ids=["block64", "block3", "window64", "full"])
@pytest.mark.parametrize("valid", [[700, 433, 64, 0, 1, 699], [700, 690, 650, 700, 600, 699]],
                         ids=["mostly-padding", "little-padding"])
def test_host_call_copies_only_valid_rows(cuda_device, mask, valid):
    """The host-buffer call copies only the rows below valid_len to the
    device, so its staging buffers keep whatever an earlier call left past
    them (NaN and Inf here).  The result must still equal the device call on
    the same inputs, bit for bit, with padded rows +0.0, for light and for
    heavy padding."""
    batch, heads, seq = 6, 3, 700
    p = oracle.Problem(batch, heads, seq, 64, **mask)
    q, k, v = oracle.qkv(p.numel, 97)
    qn, kn, vn = (x.copy().reshape(batch, heads, seq, 64) for x in (q, k, v))
    for b, vl in enumerate(valid):
        qn[b, :, vl:] = np.nan
        kn[b, :, vl:] = np.inf
        vn[b, :, vl:] = np.nan
    # an earlier call with every row valid leaves NaN/Inf in the staging rows past `valid`
    cuda_host_run(p, qn.reshape(-1), kn.reshape(-1), vn.reshape(-1), valid=[seq] * batch)
    got = cuda_host_run(p, q, k, v, valid=valid)
    want = cuda_device_run(p, q, k, v, valid=valid)
    assert np.array_equal(got, want)
    padded_rows_exact_zero(got, p, valid)


@pytest.mark.parametrize("mask", [B3, W64, dict(mask=oracle.MASK_FULL)], ids=["block3", "window64", "full"])
@pytest.mark.parametrize("kernel", [rb._lib.KERNEL_TC32_WS2, rb._lib.KERNEL_TC32_WS, rb._lib.KERNEL_TC16_WS2,
                                    rb._lib.KERNEL_TC16_WS, rb.KERNEL_AUTO])
@pytest.mark.parametrize("seq", [700, 512], ids=["seq700", "seq512"])
def test_many_units_per_sm(cuda_device, mask, kernel, seq):
    """More (slice, 128-row) units than SMs, so several CTAs run on each SM
    in turn, with padding-only units (valid 0 and short sequences) and ragged
    tails.  At seq 512 a slice is four row tiles (kernels 37 and 41 then run
    four per CTA)."""
    rng = np.random.default_rng(123)
    batch = 48 if mask is not W64 else 40
    p = oracle.Problem(batch, 4, seq, 64, **mask)
    q, k, v = oracle.qkv(p.numel, 4242)
    valid = [int(x) for x in rng.integers(0, seq + 1, size=batch)]
    valid[:4] = [0, 1, seq, 129]
    want = oracle.naive(p, q, k, v, valid)
    got = cuda_device_run(p, q, k, v, valid=valid, kernel=kernel)
    assert_close(got, want, f"kernel {kernel}")
    padded_rows_exact_zero(got, p, valid)
