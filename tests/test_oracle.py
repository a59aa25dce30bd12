"""The CPU oracle against the reference's golden vectors and known answers.

Pins the C restatement before any CUDA result is compared with it:
goldens.rs (Laya block_local golden), oracle.rs (dense reference cases),
masking.rs (mask exactness, exact-zero padding, extreme logits),
masks_dense.rs / masks_edges.rs (Full and Sliding), equivalence.rs (the
Tiled restatement against Naive, thread-count invariance).
"""
import numpy as np
import pytest

import oracle
from _util import load_golden

B3 = dict(mask=oracle.MASK_BLOCK, block=128, halo=1)
W64 = dict(mask=oracle.MASK_WINDOW, window=64)


def test_golden_pins_the_oracle():
    """goldens.rs:35-80: Naive and Tiled vs both golden tensors at 1e-5."""
    meta, g = load_golden()
    assert meta["pattern"] == "block_local"
    assert meta["scale"] == "1/sqrt(head_dim)"
    assert meta["block"] == 128
    p = oracle.Problem(1, len(meta["heads_kept"]), meta["length"], meta["head_dim"], **B3)
    q, k, v = (np.ascontiguousarray(g[n].reshape(-1)) for n in ("q", "k", "v"))
    naive = oracle.naive(p, q, k, v)
    tiled = oracle.tiled(p, q, k, v, threads=2)
    for name, got in (("naive", naive), ("tiled", tiled)):
        for gname in ("reference", "kernel"):
            diff = np.abs(got - g[gname].reshape(-1)).max()
            assert diff < meta["tolerance"], f"{name} vs golden {gname}: {diff}"
    # the restated scalar oracle reproduces the golden's reference to ~ulp level
    assert np.abs(naive - g["reference"].reshape(-1)).max() < 1e-6


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
def test_naive_matches_dense_reference(mask):
    """oracle.rs:8-32 at 1e-6 (fp64 dense reference here)."""
    for seq in [1, 7, 127, 128, 129, 257]:
        for heads, d in [(1, 8), (3, 64)]:
            for valid in [seq, max(seq - 37, 0), seq // 2]:
                p = oracle.Problem(1, heads, seq, d, **mask)
                q, k, v = oracle.qkv(p.numel, 11 + seq)
                got = oracle.naive(p, q, k, v, [valid])
                want = oracle.dense_reference(p, q, k, v, [valid])
                diff = np.abs(got - want).max() if got.size else 0.0
                assert diff < 1e-6, f"seq {seq} valid {valid} h{heads} d{d}: {diff}"


@pytest.mark.parametrize("block", [1, 7, 32, 64, 256])
@pytest.mark.parametrize("halo", [0, 1, 2])
def test_generalised_block_masks_match_dense(block, halo):
    p = oracle.Problem(3, 2, 300, 16, mask=oracle.MASK_BLOCK, block=block, halo=halo)
    q, k, v = oracle.qkv(p.numel, 5 + block)
    valid = [300, 201, 1]
    got = oracle.naive(p, q, k, v, valid)
    want = oracle.dense_reference(p, q, k, v, valid)
    assert np.abs(got - want).max() < 1e-6


def test_full_and_sliding_match_dense_softmax():
    """masks_dense.rs:49-77 and masks_edges.rs:42-72."""
    cases = []
    for w in (8, 0, 500):
        cases += [(dict(mask=oracle.MASK_WINDOW, window=w), 2, s, 16, vl) for s, vl in ((40, 40), (40, 23), (3, 1))]
    cases += [(dict(mask=oracle.MASK_FULL), 2, s, 16, vl) for s, vl in ((40, 40), (40, 23), (3, 1))]
    cases += [(dict(mask=oracle.MASK_WINDOW, window=64), 2, 200, 64, 200),
              (dict(mask=oracle.MASK_WINDOW, window=64), 2, 200, 64, 131),
              (dict(mask=oracle.MASK_WINDOW, window=64), 1, 64, 64, 64),
              (dict(mask=oracle.MASK_WINDOW, window=64), 1, 65, 32, 65),
              (dict(mask=oracle.MASK_FULL), 2, 150, 64, 150)]
    for mask, heads, seq, d, valid in cases:
        p = oracle.Problem(1, heads, seq, d, **mask)
        q, k, v = (oracle.lcg_fill(p.numel, s) for s in (1, 2, 3))
        got = oracle.naive(p, q, k, v, [valid])
        want = oracle.dense_reference(p, q, k, v, [valid])
        assert np.abs(got - want).max() < 1e-5, (mask, seq, valid)


def test_sliding_window_edges():
    """masks_dense.rs:100-106."""
    p = oracle.Problem(1, 1, 40, 8, mask=oracle.MASK_WINDOW, window=8)
    assert oracle.key_range(p, 2, 40) == (0, 11)
    assert oracle.key_range(oracle.Problem(1, 1, 7, 8, mask=oracle.MASK_FULL), 5, 7) == (0, 7)
    allowed = oracle.allowed_matrix(p, 40)
    assert allowed[20, 12] and allowed[20, 28]
    assert not allowed[20, 11] and not allowed[20, 29]


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
def test_oracle_masks_are_exact(mask):
    """masking.rs:20-61 on the oracle itself."""
    n = 300
    p = oracle.Problem(1, 1, n, 8, **mask)
    q, k = oracle.rand_vec(p.numel, 5), oracle.rand_vec(p.numel, 6)
    allowed = oracle.allowed_matrix(p, n)
    for j in [0, 1, 63, 64, 65, 127, 128, 129, 191, 255, 256, 299]:
        v = np.zeros(p.numel, dtype=np.float32)
        v[j * 8] = 1.0
        for out in (oracle.naive(p, q, k, v), oracle.tiled(p, q, k, v, threads=2)):
            w = out.reshape(n, 8)[:, 0]
            assert (w[allowed[:, j]] > 0).all()
            assert (w[~allowed[:, j]] == 0.0).all()


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
def test_oracle_padding_is_exact_zero(mask):
    """masking.rs:63-91."""
    p = oracle.Problem(1, 2, 200, 16, **mask)
    q, k, v = oracle.qkv(p.numel, 9)
    for valid in (0, 1, 150):
        for out in (oracle.naive(p, q, k, v, [valid]), oracle.tiled(p, q, k, v, [valid], threads=2)):
            o = out.reshape(2, 200, 16)
            assert (o[:, valid:] == 0.0).all() and np.isfinite(o).all()


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
def test_oracle_extreme_logits(mask):
    """masking.rs:93-126."""
    p = oracle.Problem(1, 2, 300, 64, **mask)
    q, k, v = oracle.qkv(p.numel, 21)
    q, k = q * np.float32(400), k * np.float32(400)
    want = oracle.naive(p, q, k, v)
    got = oracle.tiled(p, q, k, v, threads=2)
    assert np.isfinite(want).all() and np.isfinite(got).all()
    assert np.abs(got - want).max() < 1e-5


@pytest.mark.parametrize("mask", [B3, W64], ids=["block3", "window64"])
def test_tiled_restatement_matches_naive(mask):
    """equivalence.rs:29-66 (both backends)."""
    for seq, valid in [(1, 1), (127, 127), (129, 129), (1000, 1000), (300, 263), (256, 1), (256, 0)]:
        p = oracle.Problem(1, 2, seq, 64, **mask)
        q, k, v = oracle.qkv(p.numel, 100 + seq)
        want = oracle.naive(p, q, k, v, [valid])
        for backend in (0, 1):
            got = oracle.tiled(p, q, k, v, [valid], threads=1, backend=backend)
            assert np.abs(got - want).max() < 1e-5, (seq, valid, backend)


def test_tiled_thread_count_does_not_change_results():
    """equivalence.rs:114-129."""
    for mask in (B3, W64):
        p = oracle.Problem(1, 4, 700, 64, **mask)
        q, k, v = oracle.qkv(p.numel, 800)
        one = oracle.tiled(p, q, k, v, [650], threads=1)
        four = oracle.tiled(p, q, k, v, [650], threads=4)
        assert np.array_equal(one, four)


def test_pair_count_matches_the_allowed_matrix():
    for mask in (dict(mask=oracle.MASK_BLOCK, block=64, halo=1), dict(mask=oracle.MASK_BLOCK, block=32, halo=0),
                 W64, dict(mask=oracle.MASK_FULL)):
        p = oracle.Problem(3, 2, 257, 8, **mask)
        valid = [257, 100, 0]
        pairs, rows = oracle.count(p, valid)
        want = sum(int(oracle.allowed_matrix(p, vl).sum()) for vl in valid) * 2
        assert pairs == want and rows == 2 * sum(valid)


def test_reference_generators():
    """tests/common/mod.rs:6-18 and masks_edges.rs:6-14 known values."""
    x = oracle.rand_vec(1000, 42)
    assert x.min() >= -1 and x.max() <= 1 and abs(float(x.mean())) < 0.1
    # xorshift first value for seed 1, computed by hand from the recurrence
    s = (1 * 0x9E3779B97F4A7C15) & (2**64 - 1) | 1
    s ^= (s << 13) & (2**64 - 1)
    s ^= s >> 7
    s ^= (s << 17) & (2**64 - 1)
    want = np.float32(2.0) * (np.float32(s >> 40) / np.float32(1 << 24)) - np.float32(1.0)
    assert oracle.rand_vec(1, 1)[0] == want
    y = oracle.lcg_fill(3, 11)
    s = 11
    for i in range(3):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        assert y[i] == np.float32(s >> 8) / np.float32(1 << 24) - np.float32(0.5)
