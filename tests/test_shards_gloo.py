"""Multi-rank host logic of the sharded path, as gloo ranks on CPU.

world_size 2 processes (spawned) run the same code the GPU ranks run:
partition by raya_attn_shard, re-express the range as an independent call,
gather the shards to rank 0.  The compute step is the CPU oracle here (no GPU
in this test); the test checks the partition and reassembly bit for bit, and
that a rank which leaves before the gather makes rank 0's gather fail with
an error instead of hanging (failure detection on the host).
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    import raya_b200 as rb

    shape = rb.AttnShape(heads=3, seq=300, head_dim=16, batch=4)
    params = rb.AttnParams.new(rb.Mask.block(1), [300, 17, 256, 129], 16, block=64)
    return shape, params


def _oracle_slices(shape, params, begin, end, q, k, v):
    import oracle
    from raya_b200.shards import shard_problem

    sub_shape, sub_params = shard_problem(shape, params, begin, end)
    n = shape.seq * shape.head_dim
    p = oracle.Problem(sub_shape.batch, 1, shape.seq, shape.head_dim, mask=oracle.MASK_BLOCK,
                       block=params.block, halo=params.mask.param)
    sl = slice(begin * n, end * n)
    return oracle.naive(p, q[sl].copy(), k[sl].copy(), v[sl].copy(), sub_params.valid_len)


def _worker(rank, world, port, outdir, leave_early):
    import sys
    from datetime import timedelta

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist

    import oracle
    from raya_b200.shards import gather_to_rank0, plan

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    shape, params = _problem()
    q, k, v = oracle.qkv(shape.numel(), 3)
    sp = plan(shape, params, world)
    b, e = sp.range(rank)
    local = torch.from_numpy(_oracle_slices(shape, params, b, e, q, k, v))
    if leave_early and rank == 1:
        os._exit(0)  # leaves between steps, before the gather
    try:
        full = gather_to_rank0(local, sp, rank)
        if rank == 0:
            np.save(os.path.join(outdir, "gathered.npy"), full.numpy())
    except Exception as err:  # noqa: BLE001 - reported to the test
        with open(os.path.join(outdir, f"error{rank}.txt"), "w") as f:
            f.write(f"{type(err).__name__}: {err}")
    finally:
        if not leave_early:
            dist.destroy_process_group()


def test_two_ranks_partition_and_gather_bit_exact(tmp_path):
    import oracle

    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path), False), nprocs=2, start_method="spawn")
    got = np.load(tmp_path / "gathered.npy")
    shape, params = _problem()
    q, k, v = oracle.qkv(shape.numel(), 3)
    p = oracle.Problem(shape.batch, shape.heads, shape.seq, shape.head_dim, mask=oracle.MASK_BLOCK,
                       block=params.block, halo=1)
    want = oracle.naive(p, q, k, v, params.valid_len)
    assert np.array_equal(got, want)


def test_a_rank_that_leaves_makes_the_gather_fail_not_hang(tmp_path):
    port = _free_port()
    try:
        mp.start_processes(_worker, args=(2, port, str(tmp_path), True), nprocs=2, start_method="spawn")
    except mp.ProcessExitedException:
        pass
    err = tmp_path / "error0.txt"
    assert err.exists(), "rank 0's gather should have raised after rank 1 left"
    assert not (tmp_path / "gathered.npy").exists()


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_problems_reassemble_the_whole_call(world):
    """Single-process check of the same reassembly for more ranks."""
    import oracle
    from raya_b200.shards import plan

    shape, params = _problem()
    q, k, v = oracle.qkv(shape.numel(), 4)
    sp = plan(shape, params, world)
    parts = [_oracle_slices(shape, params, *sp.range(r), q, k, v) for r in range(world)]
    p = oracle.Problem(shape.batch, shape.heads, shape.seq, shape.head_dim, mask=oracle.MASK_BLOCK,
                       block=params.block, halo=1)
    assert np.array_equal(np.concatenate(parts), oracle.naive(p, q, k, v, params.valid_len))
