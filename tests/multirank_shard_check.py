"""Rank program for tests/test_gpu_shard.py::test_reduce_sharded_on_two_gpus (run under torchrun).

Each rank holds its slice of axis 0 of a seeded tensor on its own GPU, runs
matrix_b200.shard.reduce_sharded (local kernels, NCCL all-gather, ordered merge) for every op over the
sharded axis and over a local axis, and checks the result against the oracle's reduction of the whole
tensor.  Prints "rank ok" on success; any mismatch raises.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from matrix_b200 import backend  # noqa: E402
from matrix_b200.shard import reduce_sharded, shard_range  # noqa: E402
from oracle import oracle  # noqa: E402
from tests.helpers import assert_bits_equal, assert_sum_close  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    backend.init(local_rank)
    port = oracle.port()
    try:
        rng = np.random.default_rng(7)
        for dtype in (np.float32, np.int32):
            shape = (9, 257, 65)
            if dtype == np.float32:
                x = (np.floor(rng.standard_normal(shape) * 4) / 4).astype(np.float32)
                x[1, 3, :] = np.nan
            else:
                x = rng.integers(-(1 << 30), 1 << 30, shape, dtype=np.int32)
            lo, hi = shard_range(shape[0], world, rank)
            xd = torch.from_numpy(np.ascontiguousarray(x[lo:hi])).to(dev)
            for op in ("sum", "max", "min", "argmax", "argmin"):
                for axis in (0, 2):
                    got = reduce_sharded(op, xd, axis, shape[0])
                    if op in ("argmax", "argmin") and axis == 0:
                        got = got[1]
                    torch.cuda.synchronize()
                    want = port.reduce(op, x, axis)
                    if axis != 0:
                        want = want[lo:hi]
                    g = got.cpu().numpy()
                    tag = f"rank {rank} {op} axis {axis} {np.dtype(dtype).name}"
                    if op == "sum" and dtype == np.float32:
                        xx = (x if axis == 0 else x[lo:hi]).astype(np.float64)
                        assert_sum_close(g, want, np.abs(xx).sum(axis), tag, exact=xx.sum(axis))
                    else:
                        assert_bits_equal(g, want, tag)
        print("rank ok", flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
