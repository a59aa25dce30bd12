"""The allocation-free packed call, checked against the workspace one.

raya_attn_forward_packed_noalloc serves callers that cannot allocate device
memory (a serving runtime that owns the GPU's memory through its own pool, a
binding that only holds raw device pointers from its host, a latency-bound
loop where cudaMalloc must not run): its rotary table is a built-in device
array of 8192 positions instead of a caller workspace.  Called through the C
ABI, it must give what raya_attn_forward_packed gives with a workspace, on
two calls in a row (the second with another rotary base and a shorter
sequence, so that the array still holds the first call's table beyond it),
within the parity tolerance of the other tests.  This file is collected last.
"""
import ctypes

import numpy as np
import pytest

import oracle
import raya_b200 as rb
from raya_b200 import _lib
from _util import assert_close

pytestmark = pytest.mark.gpu


def _both(batch, seq, heads, theta, seed, block=128, halo=1):
    import torch

    dev = torch.device("cuda", 0)
    mask = rb.Mask.block(halo)
    valid = [seq] + [max(1, seq - 37 * (i + 1)) for i in range(batch - 1)]
    shape = rb.AttnShape(heads=heads, seq=seq, head_dim=64, batch=batch)
    params = rb.AttnParams.new(mask, valid, 64, block=block)
    qkv = torch.from_numpy(oracle.rand_vec(batch * seq * 3 * heads * 64, seed)).to(dev)
    dvalid = torch.tensor(valid, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    d = rb.make_desc(shape, params)

    want = torch.full((batch * seq * heads * 64,), 7.0, device=dev)
    need = ctypes.c_size_t()
    assert _lib.lib.raya_attn_packed_workspace(ctypes.byref(d), ctypes.c_float(theta), ctypes.byref(need)) == 0
    ws = torch.empty(need.value // 4, dtype=torch.float32, device=dev)
    st = _lib.lib.raya_attn_forward_packed(ctypes.byref(d), qkv.data_ptr(), want.data_ptr(), dvalid.data_ptr(),
                                           ctypes.c_float(theta), ws.data_ptr(), need.value,
                                           ctypes.c_void_p(stream))
    assert st == 0, _lib.last_error()

    got = torch.full_like(want, -3.0)
    st = _lib.lib.raya_attn_forward_packed_noalloc(ctypes.byref(d), qkv.data_ptr(), got.data_ptr(),
                                                   dvalid.data_ptr(), ctypes.c_float(theta),
                                                   ctypes.c_void_p(stream))
    assert st == 0, _lib.last_error()
    assert _lib.lib.raya_attn_sync_status(ctypes.c_void_p(stream)) == 0, _lib.last_error()
    return got.cpu().numpy(), want.cpu().numpy()


def test_noalloc_matches_the_workspace_call_on_two_calls_in_a_row(cuda_device):
    got1, want1 = _both(batch=2, seq=4096, heads=3, theta=10000.0, seed=101)
    assert np.isfinite(got1).all()
    assert_close(got1, want1, "first call")
    # second call: another base and a shorter sequence; the built-in table
    # still holds the first call's angles past position 700
    got2, want2 = _both(batch=3, seq=700, heads=2, theta=160000.0, seed=202, block=64)
    assert np.isfinite(got2).all()
    assert_close(got2, want2, "second call")


def test_noalloc_rejects_sequences_past_its_table(cuda_device):
    shape = rb.AttnShape(heads=1, seq=8193, head_dim=64, batch=1)
    d = rb.make_desc(shape, rb.AttnParams.new(rb.Mask.BLOCK3, 8193, 64))
    st = _lib.lib.raya_attn_forward_packed_noalloc(ctypes.byref(d), 16, 16, None, ctypes.c_float(10000.0), None)
    assert st == _lib.ERR_UNSUPPORTED
    assert "8192" in _lib.last_error()


def test_noalloc_at_the_table_limit_and_without_rotation_past_it(cuda_device):
    """seq exactly 8192 with the rotation (the whole built-in table in use),
    and rope_theta 0 at a seq past 8192 (no table, no limit), each against
    the workspace call."""
    got, want = _both(batch=1, seq=8192, heads=1, theta=10000.0, seed=303)
    assert np.isfinite(got).all()
    assert_close(got, want, "seq 8192 with rotation")
    got, want = _both(batch=1, seq=8192 + 300, heads=1, theta=0.0, seed=404)
    assert np.isfinite(got).all()
    assert_close(got, want, "seq 8492 without rotation")
