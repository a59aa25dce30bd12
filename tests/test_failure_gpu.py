"""Failure detection on the GPU without a fault (device-side bounded waits).

Every wait of the kernels on an mbarrier is bounded: after the limit the
kernel records a timeout in the library's status word and returns.  The
probe here waits on a barrier that nothing ever arrives on, with a short
limit; the host must read RAYA_ATTN_ERR_TIMEOUT, the record must clear, and
the context must stay usable for the next attention call."""
import ctypes

import numpy as np
import pytest

import oracle
import raya_b200 as rb
from raya_b200 import _lib
from _util import assert_close, cuda_device_run

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_reports_timeout_and_the_context_survives(cuda_device):
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    st = _lib.lib.raya_attn_probe_timeout(2_000_000, ctypes.c_void_p(stream))  # ~1 ms of cycles
    assert st == _lib.ERR_TIMEOUT, _lib.last_error()
    assert "timeout" in _lib.last_error()
    # the record was cleared by the report
    rb.sync_status()
    # and the context still runs attention correctly
    p = oracle.Problem(1, 2, 200, 64, mask=oracle.MASK_BLOCK, block=64, halo=1)
    q, k, v = oracle.qkv(p.numel, 3)
    assert_close(cuda_device_run(p, q, k, v), oracle.naive(p, q, k, v), "after timeout")


def test_probe_rejects_unbounded_limits(cuda_device):
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.raya_attn_probe_timeout(-1, ctypes.c_void_p(stream)) == _lib.ERR_SHAPE
    assert _lib.lib.raya_attn_probe_timeout(1 << 40, ctypes.c_void_p(stream)) == _lib.ERR_SHAPE
