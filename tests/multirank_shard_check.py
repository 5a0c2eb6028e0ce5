"""Rank program for tests/test_gpu_shard.py::test_reduce_sharded_on_two_gpus (run under torchrun).

Each rank holds its slice of axis 0 of a seeded tensor on its own GPU and reduces it over the sharded
axis and over a local axis, twice: through the C ABI's communicator (shard.NativeComm +
mtxc_reduce_sharded: local kernels, NCCL all-gather and ordered merge in one call) and through
torch.distributed's all-gather with the same merge kernel.  Every result is checked against the
oracle's reduction of the whole tensor.  The tensors include ArgMax / ArgMin ties that straddle the
shard boundary (the first global index must win: Matrix.mm:16291-16299), a column whose only extreme
sits at the first row of the second shard, constant columns (index 0), NaNs, and int32 sums that wrap.
mtxc_allreduce (sum / max / min) is checked against numpy on the gathered buffers.  Each rank prints which
exchange the communicator uses ("peer=1": one kernel over NVLink peer memory; "peer=0": NCCL all-gather +
merge, e.g. with MTXC_COMM_PEER=0) and "rank ok" on success; any mismatch raises.

With MTXC_SHARD_CHECK_TIMEOUT=1 the program instead checks the peer exchange's bounded wait: rank 1 skips
one exchange that rank 0 makes, so rank 0's wait for rank 1 runs out (MTXC_COMM_SPIN_LIMIT keeps that short),
the kernel returns, and mtxc_comm_status reports it; rank 0 prints "timeout reported".  No GPU hangs or
faults: the wait is bounded and nothing is read or written out of bounds.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from matrix_b200 import backend  # noqa: E402
from matrix_b200.shard import NativeComm, reduce_sharded, shard_range  # noqa: E402
from oracle import oracle  # noqa: E402
from tests.helpers import assert_bits_equal, assert_sum_close  # noqa: E402


def tensors(world):
    rng = np.random.default_rng(7)
    shape = (9, 257, 65)
    b = shard_range(shape[0], world, 1)[0] if world > 1 else 4  # first row of the second shard
    xf = (np.floor(rng.standard_normal(shape) * 4) / 4).astype(np.float32)
    xf[1, 3, :] = np.nan
    xf[b - 1, :, 0] = 100.0       # equal maxima either side of the boundary: the earlier row wins
    xf[b, :, 0] = 100.0
    xf[b, :, 1] = -100.0          # the only minimum at the second shard's first row
    xf[:, :, 2] = 1.5             # constant column: index 0
    xf[b, :, 3] = -0.0            # signed zeros across the boundary
    xf[:b, :, 3] = 0.0
    xf[b + 1:, :, 3] = -0.0
    xi = rng.integers(-(1 << 30), 1 << 30, shape, dtype=np.int32)
    xi[:, :, 5] = (1 << 30) + 7   # 9 (2^30 + 7) wraps in int32
    xi[b - 1, :, 6] = xi[b, :, 6] = np.iinfo(np.int32).max
    xi[b - 1, :, 7] = xi[b, :, 7] = np.iinfo(np.int32).min
    return shape, [xf, xi]


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    backend.init(local_rank)
    port = oracle.port()
    comm = NativeComm()
    try:
        assert (comm.world, comm.rank) == (world, rank)
        peer, _ = comm.status(wait=False)
        print(f"rank {rank} peer={int(peer)}", flush=True)
        if os.environ.get("MTXC_SHARD_CHECK_TIMEOUT") == "1":
            assert peer, "the timeout check needs the peer exchange"
            x = torch.arange(4096, dtype=torch.float32, device=dev).reshape(1, 4096)
            got = reduce_sharded("sum", x, 0, world, comm=comm)  # both ranks: completes
            torch.cuda.synchronize()
            assert comm.status() == (True, False)
            if rank == 0:
                import time

                t0 = time.perf_counter()
                reduce_sharded("sum", x, 0, world, comm=comm)  # rank 1 never makes this call
                status = comm.status()
                print(f"rank 0 waited {time.perf_counter() - t0:.3f} s, status {status}", flush=True)
                assert status == (True, True), "a wait that ran out must be reported"
                print("timeout reported", flush=True)
            assert got.shape == (4096,)
            print("rank ok", flush=True)
            return
        shape, xs = tensors(world)
        for x in xs:
            lo, hi = shard_range(shape[0], world, rank)
            xd = torch.from_numpy(np.ascontiguousarray(x[lo:hi])).to(dev)
            for op in ("sum", "max", "min", "argmax", "argmin"):
                for axis in (0, 2):
                    for path in ("native", "torch"):
                        got = reduce_sharded(op, xd, axis, shape[0], comm=comm if path == "native" else None)
                        if op in ("argmax", "argmin") and axis == 0 and path == "torch":
                            got = got[1]
                        torch.cuda.synchronize()
                        want = port.reduce(op, x, axis)
                        if axis != 0:
                            want = want[lo:hi]
                        g = got.cpu().numpy()
                        tag = f"rank {rank} {path} {op} axis {axis} {x.dtype.name}"
                        if op == "sum" and x.dtype == np.float32:
                            xx = (x if axis == 0 else x[lo:hi]).astype(np.float64)
                            assert_sum_close(g, want, np.abs(xx).sum(axis), tag, exact=xx.sum(axis))
                        else:
                            assert_bits_equal(g, want, tag)
        # mtxc_allreduce: every rank contributes its own values; the result is the rank-order merge
        rng = np.random.default_rng(11)
        allv = rng.integers(-(1 << 31), (1 << 31) - 1, (world, 1000), dtype=np.int64).astype(np.int32)
        for op, fn in (("sum", None), ("max", np.max), ("min", np.min)):
            buf = torch.from_numpy(allv[rank].copy()).to(dev)
            backend.allreduce(op, buf)
            torch.cuda.synchronize()
            want = allv.astype(np.int64).sum(0).astype(np.int32) if fn is None else fn(allv, axis=0)
            assert_bits_equal(buf.cpu().numpy(), want, f"rank {rank} allreduce {op}")
        print("rank ok", flush=True)
    finally:
        torch.cuda.synchronize()
        dist.barrier()      # every rank's kernels are done before any rank unmaps or frees its buffers
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
