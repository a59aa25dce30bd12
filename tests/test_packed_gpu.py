"""The caller's layout, fused (raya_attn_forward_packed), on a B200.

raya's encoder (crates/raya-core/src/encoder.rs:57-92) splits a packed
[seq][3][heads][head_dim] projection into head-major q, k, v, applies its
rotary embedding (ops.rs:110-141) to q and k, calls the kernel, and
transposes the output back to [seq][heads*head_dim].  The fused call does all
of that in the attention kernel; it is checked against the oracle's
restatement of exactly those steps (oracle.encoder_attend).
"""
import numpy as np
import pytest

import oracle
import raya_b200 as rb
from _util import assert_close

pytestmark = pytest.mark.gpu

MASKS = [(dict(mask=oracle.MASK_BLOCK, block=64, halo=1), rb.Mask.block(1), 64),
         (dict(mask=oracle.MASK_BLOCK, block=128, halo=1), rb.Mask.BLOCK3, 128),
         (dict(mask=oracle.MASK_BLOCK, block=64, halo=0), rb.Mask.block(0), 64),
         (dict(mask=oracle.MASK_WINDOW, window=64), rb.Mask.WINDOW64, 128),
         (dict(mask=oracle.MASK_FULL), rb.Mask.FULL, 128)]


def _run_packed(qkv, batch, seq, heads, mask, block, valid, theta):
    import torch

    dev = torch.device("cuda", 0)
    shape = rb.AttnShape(heads=heads, seq=seq, head_dim=64, batch=batch)
    params = rb.AttnParams.new(mask, valid, 64, block=block)
    t = torch.from_numpy(qkv).to(dev)
    ctx = torch.full((batch * seq * heads * 64,), 7.0, dtype=torch.float32, device=dev)
    rb.Cuda().attend_packed(shape, params, t, ctx, rope_theta=theta)
    rb.sync_status()
    return ctx.cpu().numpy()


@pytest.mark.parametrize("theta", [None, 10000.0, 160000.0], ids=["no-rope", "rope1e4", "rope1.6e5"])
@pytest.mark.parametrize("case", range(len(MASKS)), ids=["block64", "block3", "own64", "window64", "full"])
def test_packed_layout_matches_split_rope_attend_merge(cuda_device, case, theta):
    okw, mask, block = MASKS[case]
    batch, seq, heads = 3, 700, 4
    valid = [700, 433, 64]
    qkv = oracle.rand_vec(batch * seq * 3 * heads * 64, 55 + case)
    want = oracle.encoder_attend(qkv, batch, seq, heads, 64, okw["mask"], okw.get("block", 128),
                                 okw.get("halo", 1), okw.get("window", 64), valid, theta)
    got = _run_packed(qkv, batch, seq, heads, mask, block, valid, theta)
    assert_close(got, want, f"packed theta={theta}")
    c = got.reshape(batch, seq, heads * 64)
    for b, vl in enumerate(valid):
        assert (c[b, vl:] == 0.0).all()


@pytest.mark.parametrize("theta", [None, 10000.0], ids=["no-rope", "rope1e4"])
@pytest.mark.parametrize("case", [0, 1, 3], ids=["block64", "block3", "window64"])
def test_packed_layout_edge_valid_lengths(cuda_device, case, theta):
    """A sequence with nothing valid, one with a single valid row and one a row
    past a 128-row tile: exact zeros past valid_len, the oracle's values below."""
    okw, mask, block = MASKS[case]
    batch, seq, heads = 3, 300, 2
    valid = [0, 1, 129]
    qkv = oracle.rand_vec(batch * seq * 3 * heads * 64, 91 + case)
    want = oracle.encoder_attend(qkv, batch, seq, heads, 64, okw["mask"], okw.get("block", 128),
                                 okw.get("halo", 1), okw.get("window", 64), valid, theta)
    got = _run_packed(qkv, batch, seq, heads, mask, block, valid, theta)
    assert_close(got, want, f"packed edge theta={theta}")
    c = got.reshape(batch, seq, heads * 64)
    for b, vl in enumerate(valid):
        assert (c[b, vl:] == 0.0).all() and not np.signbit(c[b, vl:]).any()


# (batch, seq, heads, valid): 48 row tiles (one tile per CTA), and 1024 row
# tiles at block 64 (two tiles per CTA, the form the automatic choice takes).
BIG = (8, 512, 32, [512, 300, 257, 256, 511, 129, 0, 400])


@pytest.mark.parametrize("dims", [(2, 1000, 3, [1000, 511]), BIG], ids=["48-tiles", "1024-tiles"])
def test_packed_layout_equals_the_head_major_call_bit_for_bit(cuda_device, dims):
    """Without rotation the fused layout only changes addressing: the result is
    the head-major call's with the same kernel, transposed, bit for bit."""
    import torch

    batch, seq, heads, valid = dims
    qkv = oracle.rand_vec(batch * seq * 3 * heads * 64, 9)
    got = _run_packed(qkv, batch, seq, heads, rb.Mask.block(1), 64, valid, None)
    x = qkv.reshape(batch, seq, 3, heads, 64)
    q, k, v = (np.ascontiguousarray(x[:, :, w].transpose(0, 2, 1, 3)).reshape(-1) for w in range(3))
    shape = rb.AttnShape(heads=heads, seq=seq, head_dim=64, batch=batch)
    params = rb.AttnParams.new(rb.Mask.block(1), valid, 64, block=64)
    dev = torch.device("cuda", 0)
    tq, tk, tv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    out = torch.empty_like(tq)
    rb.Cuda().attend_device(shape, params, tq, tk, tv, out, kernel=rb.kernel_for(shape, params, packed=True))
    rb.sync_status()
    head_major = out.cpu().numpy().reshape(batch, heads, seq, 64).transpose(0, 2, 1, 3).reshape(-1)
    assert np.array_equal(got, head_major)


@pytest.mark.parametrize("theta", [None, 10000.0], ids=["no-rope", "rope1e4"])
def test_packed_layout_with_many_row_tiles_matches_the_oracle(cuda_device, theta):
    """Enough row tiles for two per CTA (the form taken without rotation; with
    it, one per CTA), ragged and empty sequences among them."""
    batch, seq, heads, valid = BIG
    assert rb.kernel_for(rb.AttnShape(heads=heads, seq=seq, head_dim=64, batch=batch),
                         rb.AttnParams.new(rb.Mask.block(1), valid, 64, block=64), packed=True,
                         rope=theta is not None) == (rb._lib.KERNEL_TC32_WS2 if theta is None else rb._lib.KERNEL_TC32_WS)
    qkv = oracle.rand_vec(batch * seq * 3 * heads * 64, 13)
    want = oracle.encoder_attend(qkv, batch, seq, heads, 64, oracle.MASK_BLOCK, 64, 1, 64, valid, theta)
    got = _run_packed(qkv, batch, seq, heads, rb.Mask.block(1), 64, valid, theta)
    assert_close(got, want, f"packed two tiles theta={theta}")
    c = got.reshape(batch, seq, heads * 64)
    for b, vl in enumerate(valid):
        assert (c[b, vl:] == 0.0).all() and not np.signbit(c[b, vl:]).any()


def test_long_positions_rotate_like_the_reference(cuda_device):
    """Rotary angles grow with the position: seq 8192 checks the f32 angle path."""
    batch, seq, heads = 1, 8192, 2
    qkv = oracle.rand_vec(batch * seq * 3 * heads * 64, 77)
    want = oracle.encoder_attend(qkv, batch, seq, heads, 64, oracle.MASK_BLOCK, 128, 1, 64, [seq], 10000.0)
    got = _run_packed(qkv, batch, seq, heads, rb.Mask.BLOCK3, 128, [seq], 10000.0)
    assert_close(got, want, "seq 8192 rope")
