"""Batch x heads sharding over real GPUs (needs 2+ GPUs; skipped otherwise).

Two ranks (one process per GPU, NCCL) each take their range of slices from
raya_attn_shard, run the CUDA kernel on it as an independent call, and gather
the outputs to rank 0 over NVLink; rank 0 compares with one single-GPU call
over the whole batch: the result must be identical bit for bit (slices are
independent, so sharding cannot change any rounding).  NVLS is off and no
kernel here uses multimem or TMA multicast.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    import raya_b200 as rb

    shape = rb.AttnShape(heads=12, seq=1024, head_dim=64, batch=6)
    params = rb.AttnParams.new(rb.Mask.block(1), [1024, 700, 512, 1, 999, 0], 64, block=64)
    return shape, params


def _worker(rank, world, port, outdir):
    import sys
    from datetime import timedelta

    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    import oracle
    import raya_b200 as rb
    from raya_b200.shards import gather_to_rank0, plan, shard_problem

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        shape, params = _problem()
        q, k, v = oracle.qkv(shape.numel(), 17)
        sp = plan(shape, params, world)
        b, e = sp.range(rank)
        n = shape.seq * shape.head_dim
        sub_shape, sub_params = shard_problem(shape, params, b, e)
        tq, tk, tv = (torch.from_numpy(x[b * n:e * n].copy()).to(dev) for x in (q, k, v))
        out = torch.empty((e - b) * n, dtype=torch.float32, device=dev)
        if e > b:
            rb.Cuda(rb.CudaConfig(device=rank)).attend_device(sub_shape, sub_params, tq, tk, tv, out)
            rb.sync_status()
        full = gather_to_rank0(out, sp, rank)
        if rank == 0:
            np.save(os.path.join(outdir, "gathered.npy"), full.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_shards_gather_to_the_single_gpu_result(tmp_path):
    import torch

    import oracle
    import raya_b200 as rb

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, start_method="spawn")
    got = np.load(tmp_path / "gathered.npy")
    shape, params = _problem()
    q, k, v = oracle.qkv(shape.numel(), 17)
    out = np.empty(shape.numel(), dtype=np.float32)
    rb.Cuda().attend(shape, params, q, k, v, out)
    assert np.array_equal(got, out)


def _multi_problem():
    import raya_b200 as rb

    shape = rb.AttnShape(heads=5, seq=900, head_dim=64, batch=7)
    params = rb.AttnParams.new(rb.Mask.block(1), [900, 1, 0, 513, 899, 640, 128], 64, block=128)
    return shape, params


@pytest.mark.parametrize("devices", [[0], [0, 1], [1, 0]], ids=["one", "two", "two-gather-on-1"])
def test_multi_gpu_entry_point_equals_the_single_gpu_call(cuda_device, devices):
    """raya_attn_forward_multi_gpu through the C ABI: slices split over the
    devices by raya_attn_shard, host output and the device-side gather on
    devices[0] both bit-identical to raya_attn_forward_host on one GPU."""
    import torch

    import oracle
    import raya_b200 as rb

    if max(devices) >= torch.cuda.device_count():
        pytest.skip(f"needs {max(devices) + 1} GPUs")
    shape, params = _multi_problem()
    q, k, v = oracle.qkv(shape.numel(), 31)
    want = np.empty(shape.numel(), dtype=np.float32)
    rb.Cuda().attend(shape, params, q, k, v, want)
    got = np.full(shape.numel(), 7.0, dtype=np.float32)
    gathered = torch.full((shape.numel(),), -3.0, dtype=torch.float32, device=torch.device("cuda", devices[0]))
    rb.multi_gpu(shape, params, q, k, v, got, devices=devices, out_device0=gathered)
    assert np.array_equal(got, want)
    assert np.array_equal(gathered.cpu().numpy(), want)
    # the device-side gather alone (no host output)
    gathered.fill_(5.0)
    rb.multi_gpu(shape, params, q, k, v, None, devices=devices, out_device0=gathered)
    assert np.array_equal(gathered.cpu().numpy(), want)
