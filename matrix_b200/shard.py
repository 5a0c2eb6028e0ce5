"""Leading-axis sharding of the hot path across the GPUs of one node (one process per GPU).

A tensor whose axis 0 has `n` entries is split into `world` contiguous slices; rank r holds
[shard_range(n, world, r)).  Elementwise ops and reductions over any other axis are local: their
results stay sharded the same way and no data crosses GPUs.  A reduction over axis 0 -- the sharded
axis -- produces one partial per rank; the partials are exchanged with an all-gather (NCCL over
NVLink on GPUs) and merged in rank order by mtxc_merge_partials, which keeps the reference's
semantics across shards (ordered sums, first shard wins ties, global first index for ArgMax /
ArgMin).  The merge runs identically on every rank, so every rank holds the same result.

The compute steps are injected (`ops`), so the bookkeeping -- slice bounds, the gather, index
offsets -- is the same code whether the partials come from the GPU kernels or from a CPU stand-in.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced slice [lo, hi) of n entries for `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return n * rank // world, n * (rank + 1) // world


def shard_offsets(n: int, world: int) -> list[int]:
    return [shard_range(n, world, r)[0] for r in range(world)]


@dataclass
class ShardOps:
    """The compute steps of a sharded reduction.

    local(op, x, axis, keepdims) -> the op's result (indices for argmax / argmin);
    local_pair(op, x, axis, keepdims) -> (extreme values, first indices) for argmax / argmin;
    merge(op, values [parts, ...], indices | None, offsets) -> values, or (values, indices).
    """
    local: Callable
    local_pair: Callable
    merge: Callable


def gpu_ops() -> ShardOps:
    from . import backend

    return ShardOps(local=lambda op, x, axis, keepdims: backend.reduce(op, x, axis, keepdims),
                    local_pair=backend.reduce_pair, merge=backend.merge_partials)


def all_gather_stacked(t: torch.Tensor, group=None) -> torch.Tensor:
    """[world, *t.shape]: every rank's tensor, in rank order."""
    world = dist.get_world_size(group)
    if world == 1:
        return t.unsqueeze(0)
    flat = t.contiguous().reshape(-1)
    out = torch.empty(world * flat.numel(), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    return out.reshape(world, *t.shape)


def reduce_sharded(op: str, x_local: torch.Tensor, axis: int, global_len: int, keepdims: bool = False,
                   group=None, ops: ShardOps | None = None):
    """x.<op>(axis, keepdims) for a tensor x sharded along axis 0 (this rank holds x_local).

    Over axis 0 the result is complete and identical on every rank; over any other axis it is this
    rank's shard of the result (sharded along axis 0 like the input)."""
    ops = ops or gpu_ops()
    dims = x_local.dim()
    ax = axis + dims if axis < 0 else axis
    if ax != 0:
        return ops.local(op, x_local, ax, keepdims)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_range(global_len, world, rank)
    if x_local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds {x_local.shape[0]} rows of axis 0, expected {hi - lo}")
    offsets = shard_offsets(global_len, world)
    if op in ("argmax", "argmin"):
        v, i = ops.local_pair(op, x_local, 0, keepdims)
        return ops.merge(op, all_gather_stacked(v, group), all_gather_stacked(i, group), offsets)
    v = ops.local(op, x_local, 0, keepdims)
    return ops.merge(op, all_gather_stacked(v, group), None, offsets)
