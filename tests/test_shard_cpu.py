"""Leading-axis sharding, host logic, on CPU ranks (gloo, world sizes 2 and 3).

matrix_b200.shard.reduce_sharded is run on CPU processes with its compute steps replaced by CPU
stand-ins: the local reductions by the oracle, the ordered merge by a NumPy statement of the merge
rule mtxc_merge_partials implements.  The slice bounds, the all-gather, the index offsets and the
rank order are the product code under test; results must equal the oracle's reduction of the whole,
unsharded tensor (bit for bit except float sums, compared with the usual tolerance).
"""
import os
import socket

import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal, assert_sum_close

OPS = ["sum", "max", "min", "argmax", "argmin"]


def numpy_merge(op, values, indices, offsets):
    """Merge rule of mtxc_merge_partials: shard order, strict comparisons, index offsets."""
    v = values.numpy()
    if op == "sum":
        acc = v[0].copy()
        for p in range(1, v.shape[0]):
            acc = (acc + v[p]).astype(v.dtype)
        return torch.from_numpy(acc)
    best, src = v[0].copy(), np.zeros(v.shape[1:], dtype=np.int64)
    for p in range(1, v.shape[0]):
        better = (best < v[p]) if op in ("max", "argmax") else (v[p] < best)
        best = np.where(better, v[p], best)
        src = np.where(better, p, src)
    if op in ("max", "min"):
        return torch.from_numpy(best)
    idx = np.take_along_axis(indices.numpy(), src[None], 0)[0] + np.asarray(offsets)[src]
    return torch.from_numpy(best), torch.from_numpy(idx.astype(np.int32))


def cpu_ops():
    from matrix_b200.shard import ShardOps
    from oracle import oracle

    port = oracle.port()

    def local(op, x, axis, keepdims):
        return torch.from_numpy(port.reduce(op, x.numpy(), axis, keepdims))

    def local_pair(op, x, axis, keepdims):
        a = x.numpy()
        return (torch.from_numpy(port.reduce(op[3:], a, axis, keepdims)),
                torch.from_numpy(port.reduce(op, a, axis, keepdims)))

    return ShardOps(local=local, local_pair=local_pair, merge=numpy_merge)


def make_global(dtype):
    rng = np.random.default_rng(42)
    shape = (11, 6, 37)
    if dtype == np.float32:
        x = (np.floor(rng.standard_normal(shape) * 8) / 8).astype(np.float32)  # ties across shards
        x[3, 2, :] = np.nan
        x[:, 4, 5] = -0.0
        x[5:, 4, 5] = 0.0
    else:
        x = rng.integers(-(1 << 30), 1 << 30, shape, dtype=np.int32)
    return x


def _worker(rank, world, port, results):
    import torch.distributed as dist

    from matrix_b200.shard import reduce_sharded, shard_range
    from oracle import oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        full_oracle = oracle.port()
        ops = cpu_ops()
        for dtype in (np.float32, np.int32):
            x = make_global(dtype)
            lo, hi = shard_range(x.shape[0], world, rank)
            local = torch.from_numpy(np.ascontiguousarray(x[lo:hi]))
            for op in OPS:
                for axis in (0, 1, 2):
                    got = reduce_sharded(op, local, axis, x.shape[0], ops=ops)
                    if op in ("argmax", "argmin") and axis == 0:
                        got_v, got = got
                        assert_bits_equal(got_v.numpy(), full_oracle.reduce(op[3:], x, 0), f"{op} value")
                    want = full_oracle.reduce(op, x, axis)
                    if axis != 0:
                        want = want[lo:hi]
                    g = got.numpy()
                    tag = f"rank {rank}/{world} {op} axis {axis} {np.dtype(dtype).name}"
                    if op == "sum" and dtype == np.float32:
                        xx = x.astype(np.float64) if axis == 0 else x[lo:hi].astype(np.float64)
                        assert_sum_close(g, want, np.abs(xx).sum(axis if axis == 0 else axis), tag,
                                         exact=xx.sum(axis))
                    else:
                        assert_bits_equal(g, want, tag)
        results[rank] = "ok"
    except BaseException as e:  # reported to the parent
        results[rank] = repr(e)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 3])
def test_reduce_sharded_on_gloo_ranks(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert dict(results) == {r: "ok" for r in range(world)}, dict(results)


def test_shard_ranges_cover_the_axis():
    from matrix_b200.shard import shard_offsets, shard_range

    for n in (0, 1, 7, 8, 11, 4096):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
            assert shard_offsets(n, world) == [s[0] for s in spans]


def _absent_rank_worker(rank, port, mode, results):
    """Rank 1 joins the group but never reaches the collective: it idles past rank 0's timeout
    ("idle") or leaves at once ("exit").  Rank 0 runs reduce_sharded and must get an error."""
    import datetime
    import time

    import torch.distributed as dist

    from matrix_b200.shard import reduce_sharded, shard_range

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        if mode == "idle":
            time.sleep(12)
        results[rank] = "left"
        return  # no destroy: the rank is gone as far as the group knows
    t0 = time.monotonic()
    try:
        lo, hi = shard_range(11, 2, 0)
        x = torch.from_numpy(make_global(np.int32)[lo:hi].copy())
        reduce_sharded("sum", x, 0, 11, ops=cpu_ops())
        results[rank] = "no error"
    except Exception as e:  # the failure the caller must see
        results[rank] = f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}: {str(e)[:200]}"


@pytest.mark.parametrize("mode", ["idle", "exit"])
def test_absent_rank_is_an_error_not_a_hang(mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_absent_rank_worker, args=(r, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p.is_alive() for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not any(alive), f"a rank hung: {dict(results)}"
    r0 = results.get(0, "")
    assert r0.startswith("error after"), dict(results)
    elapsed = float(r0.split()[2])
    assert elapsed < 30, r0
    if mode == "idle":  # the collective itself gave up: after the group's 3 s timeout, not before
        assert elapsed >= 2.5, r0
