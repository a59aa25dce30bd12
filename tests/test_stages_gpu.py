"""Stage timing (raya_attn_forward_timed), the counterpart of the reference's
StageTimes (crates/raya-kernels/src/tiled/stages.rs:1-31) and
attend_with_stages (tiled/mod.rs:60-126), on a B200.

For the tiled FFMA kernel and the tensor-core kernels (ids 34 and 37): the
timed build writes the same output as the untimed one, bit for bit; the QK,
softmax and PV counters are positive and their percentages sum to 100; the
tensor-core kernels' tile counter equals the key tiles their 128-row units
walk, counted on the host.
"""
import numpy as np
import pytest

import oracle
import raya_b200 as rb
from _util import shape_params

pytestmark = pytest.mark.gpu


def _key_tiles(p, valid, bm=128, bn=64):
    """Key tiles the tensor-core kernel's 128-row units walk."""
    total = 0
    for b in range(p.batch):
        vl = int(valid[b])
        for r0 in range(0, p.seq, bm):
            if r0 >= vl:
                continue
            last = min(r0 + bm, vl) - 1
            lo, _ = oracle.key_range(p, r0, vl)
            _, hi = oracle.key_range(p, last, vl)
            if hi > lo:
                total += (hi + bn - 1) // bn - lo // bn
    return total * p.heads


@pytest.mark.parametrize("kernel", [rb.KERNEL_TILED64, rb.KERNEL_TC32_WS, rb.KERNEL_TC32_WS2, rb.KERNEL_TC16_WS,
                                    rb.KERNEL_TC16_WS2, rb.KERNEL_AUTO])
@pytest.mark.parametrize("block,seq", [(64, 1024), (128, 2048), (64, 512)], ids=["b64", "b128", "b64-seq512"])
def test_stage_timing(cuda_device, kernel, block, seq):
    import torch

    p = oracle.Problem(3, 4, seq, 64, mask=oracle.MASK_BLOCK, block=block, halo=1)
    valid = np.array([seq, seq // 2 + 17, 1], dtype=np.int32)
    q, k, v = oracle.qkv(p.numel, 77)
    shape, params = shape_params(p, valid)
    dev = cuda_device
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    dvalid = torch.from_numpy(valid).to(dev)
    plain = torch.full((p.numel,), 7.0, device=dev)
    timed = torch.full((p.numel,), -7.0, device=dev)
    rb.Cuda().attend_device(shape, params, tq, tk, tv, plain, valid_len=dvalid, kernel=kernel)
    st = rb.stage_times(shape, params, tq, tk, tv, timed, valid_len=dvalid, kernel=kernel)
    assert torch.equal(plain, timed), "the timed build must write the untimed output"
    for name in ("qk", "softmax", "pv", "total", "tiles"):
        assert st[name] > 0, (name, st)
    assert abs(st["qk_pct"] + st["softmax_pct"] + st["pv_pct"] - 100.0) < 1e-6
    chosen = rb.kernel_for(shape, params) if kernel == rb.KERNEL_AUTO else kernel
    if chosen in (rb.KERNEL_TC32_WS, rb.KERNEL_TC32_WS2, rb.KERNEL_TC16_WS, rb.KERNEL_TC16_WS2):
        assert st["tiles"] == _key_tiles(p, valid), st
