"""Batch x heads sharding over GPUs (one process per GPU).

Block-local attention has no cross-slice dependency: every (batch entry,
head) slice reads only its own q, k, v.  So the multi-GPU path is:

  1. every rank computes the same partition (``raya_attn_shard``: contiguous
     ranges of flattened batch*heads slices, balanced by allowed-pair count);
  2. rank r generates or receives only its slices and runs the kernel on
     them as an independent call (``shard_problem``: the range re-expressed as
     ``batch = #slices, heads = 1`` with one valid length per slice);
  3. optionally the output shards are gathered to rank 0
     (``gather_to_rank0``: point-to-point receives straight into rank 0's
     output tensor, NCCL over NVLink on GPUs, gloo on CPU).

There is no collective on the compute path.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .attention import AttnParams, AttnShape, shard


@dataclass(frozen=True)
class ShardPlan:
    world: int
    ranges: tuple[tuple[int, int], ...]  # [begin, end) of flattened slices per rank
    slice_elems: int                      # seq * head_dim

    def range(self, rank: int) -> tuple[int, int]:
        return self.ranges[rank]

    def elems(self, rank: int) -> int:
        b, e = self.ranges[rank]
        return (e - b) * self.slice_elems

    @property
    def max_elems(self) -> int:
        return max(self.elems(r) for r in range(self.world))


def plan(shape: AttnShape, params: AttnParams, world: int) -> ShardPlan:
    ranges = tuple(shard(shape, params, world, r) for r in range(world))
    return ShardPlan(world=world, ranges=ranges, slice_elems=shape.seq * shape.head_dim)


def shard_problem(shape: AttnShape, params: AttnParams, begin: int, end: int):
    """The slices [begin, end) as an independent call: (shape, params)."""
    valid = params.valid_array(shape.batch)
    per_slice = np.repeat(valid, shape.heads)[begin:end]
    sub_shape = AttnShape(heads=1, seq=shape.seq, head_dim=shape.head_dim, batch=max(end - begin, 0))
    sub_params = AttnParams(mask=params.mask, block=params.block,
                            valid_len=per_slice.astype(np.int32), scale=params.scale)
    return sub_shape, sub_params


def gather_to_rank0(local, sp: ShardPlan, rank: int, group=None, out=None):
    """Gathers every rank's output shard (a 1-D tensor of sp.elems(rank)
    floats) into one tensor on rank 0, in slice order; None on other ranks.

    Rank 0's result is ``out`` (the whole output, 1-D; allocated here when
    None).  Each other rank's shard is received straight into its slice
    range of ``out`` by point-to-point transfers (NCCL over NVLink between
    GPUs, gloo on CPU), all posted at once; rank 0's own shard is copied in
    only when ``local`` is not already that range of ``out`` (a kernel can
    write it there directly).  Nothing is padded or concatenated."""
    import torch
    import torch.distributed as dist

    n = sp.slice_elems
    if rank == 0:
        total = sp.ranges[-1][1] * n
        if out is None:
            out = torch.empty(total, dtype=local.dtype, device=local.device)
        b, e = sp.range(0)
        own = out[b * n:e * n]
        if e > b and own.data_ptr() != local.data_ptr():
            own.copy_(local)
        ops = [dist.P2POp(dist.irecv, out[rb * n:re * n], r, group)
               for r, (rb, re) in enumerate(sp.ranges) if r > 0 and re > rb]
        for req in (dist.batch_isend_irecv(ops) if ops else []):
            req.wait()
        return out
    if sp.elems(rank) > 0:
        for req in dist.batch_isend_irecv([dist.P2POp(dist.isend, local, 0, group)]):
            req.wait()
    return None
