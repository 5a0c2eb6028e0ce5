"""Leading-axis sharding of the hot path across the GPUs of one node (one process per GPU).

A tensor whose axis 0 has `n` entries is split into `world` contiguous slices; rank r holds
[shard_range(n, world, r)).  Elementwise ops and reductions over any other axis are local: their
results stay sharded the same way and no data crosses GPUs.  A reduction over axis 0 -- the sharded
axis -- produces one partial per rank; the partials are exchanged with an all-gather (NCCL over
NVLink on GPUs) and merged in rank order by mtxc_merge_partials, which keeps the reference's
semantics across shards (ordered sums, first shard wins ties, global first index for ArgMax /
ArgMin).  The merge runs identically on every rank, so every rank holds the same result.

On GPUs the exchange runs inside the C ABI: `NativeComm` creates the thread's communicator
(mtxc_comm_init) and `reduce_sharded(..., comm=...)` enqueues the local reduction, the NCCL all-gather and
the merge with one call (mtxc_reduce_sharded); torch.distributed only carries the unique id from rank 0.
Without a communicator the compute steps are injected (`ops`) and the gather is torch.distributed's, so
the bookkeeping -- slice bounds, the gather, index offsets -- is the same code whether the partials come
from the GPU kernels or from a CPU stand-in (gloo ranks in the CPU tests).
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


class NativeComm:
    """The calling thread's communicator in the C ABI (mtxc_comm_init), one rank per process and GPU.

    Rank 0 draws the unique id (mtxc_comm_unique_id) and torch.distributed broadcasts it -- plumbing only;
    the exchanges themselves run in the library on the thread's stream.  backend.init must have bound
    the thread to its device first.  buffer_bytes: the gather buffer (0: the library's 16 MiB)."""

    def __init__(self, group=None, buffer_bytes: int = 0):
        import ctypes

        from . import _abi

        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        uid = ctypes.create_string_buffer(_abi.COMM_ID_BYTES)
        if self.world > 1:
            if self.rank == 0:
                _abi.check(_abi.lib().mtxc_comm_unique_id(uid, _abi.COMM_ID_BYTES))
            box = [uid.raw]
            dist.broadcast_object_list(box, src=0, group=group)
            uid = ctypes.create_string_buffer(box[0], _abi.COMM_ID_BYTES)
        _abi.check(_abi.lib().mtxc_comm_init(self.world, self.rank, uid, int(buffer_bytes)))
        self.open = True

    def status(self, wait: bool = True) -> tuple[bool, bool]:
        """(peer_exchange, timed_out): whether the exchanges run as one kernel over peer memory, and -- when
        `wait` (the thread's stream is synchronised first) -- whether an exchange since the last query gave up
        waiting for a rank."""
        import ctypes

        from . import _abi

        peer, late = ctypes.c_int(0), ctypes.c_int(0)
        _abi.check(_abi.lib().mtxc_comm_status(ctypes.byref(peer), ctypes.byref(late) if wait else None))
        return bool(peer.value), bool(late.value)

    def close(self) -> None:
        from . import _abi

        if self.open:
            _abi.check(_abi.lib().mtxc_comm_destroy())
            self.open = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


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
                   group=None, ops: ShardOps | None = None, comm: NativeComm | None = None, out=None, meta=None):
    """x.<op>(axis, keepdims) for a tensor x sharded along axis 0 (this rank holds x_local).

    Over axis 0 the result is complete and identical on every rank; over any other axis it is this
    rank's shard of the result (sharded along axis 0 like the input).  With `comm` the axis-0 case is one
    mtxc_reduce_sharded call (ArgMax / ArgMin then return the global indices only); `out` / `meta` let a
    caller that repeats the call reuse its output tensor and metadata."""
    dims = x_local.dim()
    ax = axis + dims if axis < 0 else axis
    if ax != 0:
        return (ops or gpu_ops()).local(op, x_local, ax, keepdims)
    world = comm.world if comm is not None else dist.get_world_size(group)
    rank = comm.rank if comm is not None else dist.get_rank(group)
    lo, hi = shard_range(global_len, world, rank)
    if x_local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds {x_local.shape[0]} rows of axis 0, expected {hi - lo}")
    offsets = shard_offsets(global_len, world)
    if comm is not None:
        from . import backend

        if meta is None:
            meta = backend.reduce_meta(list(x_local.shape), list(x_local.stride()), 0, keepdims)
        if out is None:
            odt = torch.int32 if op in ("argmax", "argmin") else x_local.dtype
            out = torch.empty(meta.out_shape, dtype=odt, device=x_local.device)
        backend.reduce_sharded_launch(op, x_local.data_ptr(), backend.dtype_code(x_local.dtype), out.data_ptr(), meta,
                                      offsets)
        return out
    ops = ops or gpu_ops()
    if op in ("argmax", "argmin"):
        v, i = ops.local_pair(op, x_local, 0, keepdims)
        return ops.merge(op, all_gather_stacked(v, group), all_gather_stacked(i, group), offsets)
    v = ops.local(op, x_local, 0, keepdims)
    return ops.merge(op, all_gather_stacked(v, group), None, offsets)
