"""The cross-shard kernels on one GPU, and the sharded path on real GPU ranks when there are two.

* mtxc_reduce_pair: the (Max, ArgMax) / (Min, ArgMin) pair from one read must equal the separate
  reductions (and hence the oracle) bit for bit.
* mtxc_merge_partials: a tensor is cut along axis 0 into uneven "shards" on one device, each shard
  is reduced on its own, the partials are stacked in shard order and merged; the result must equal
  the oracle's reduction of the whole tensor (bit for bit, float sums within the usual tolerance).
* With two GPUs, matrix_b200.shard.reduce_sharded runs under torchrun with NCCL and must agree with
  the oracle on every rank.
"""
import os
import re
import socket
import subprocess
import sys

import numpy as np
import pytest

from tests.helpers import assert_bits_equal, assert_sum_close, make_values

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("op", ["max", "min"])
def test_reduce_pair_equals_separate_reductions(gpu, port, op):
    import torch

    rng = np.random.default_rng(3)
    for shape, axis in (([64, 8192, 64], 1), ([33, 1000], 1), ([4, 70000], 1), ([300, 9, 40], 0), ([5, 1 << 20], 1)):
        x = make_values(rng, int(np.prod(shape)), np.float32, "ties").reshape(shape)
        x.reshape(-1)[::97] = np.nan
        xd = torch.from_numpy(x).cuda()
        v, i = gpu.reduce_pair(op, xd, axis)
        gpu.sync()
        assert_bits_equal(v.cpu().numpy(), port.reduce(op, x, axis), f"pair value {op} {shape}")
        assert_bits_equal(i.cpu().numpy(), port.reduce("arg" + op, x, axis), f"pair index {op} {shape}")


@pytest.mark.parametrize("dtype", [np.float32, np.int32, np.int64], ids=["f32", "i32", "i64"])
@pytest.mark.parametrize("op", ["sum", "max", "min", "argmax", "argmin"])
def test_merge_partials_of_simulated_shards(gpu, port, op, dtype):
    import torch

    rng = np.random.default_rng(5)
    shape = [13, 300, 70]
    if dtype == np.float32:
        x = (np.floor(rng.standard_normal(shape) * 4) / 4).astype(np.float32)
        x[2, 5, :] = np.nan
        x[:, 7, 3] = -0.0
        x[6:, 7, 3] = 0.0
        x[:, 9, :] = -np.inf
    else:
        x = make_values(rng, int(np.prod(shape)), dtype, "full").reshape(shape)
    xd = torch.from_numpy(x).cuda()
    bounds = [0, 3, 4, 9, 13]  # uneven shards along axis 0
    parts_v, parts_i = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        if op in ("argmax", "argmin"):
            v, i = gpu.reduce_pair(op, xd[lo:hi], 0)
            parts_v.append(v)
            parts_i.append(i)
        else:
            parts_v.append(gpu.reduce(op, xd[lo:hi], 0))
    vals = torch.stack(parts_v)
    if op in ("argmax", "argmin"):
        mv, mi = gpu.merge_partials(op, vals, torch.stack(parts_i), bounds[:-1])
        gpu.sync()
        assert_bits_equal(mi.cpu().numpy(), port.reduce(op, x, 0), f"merged {op}")
        assert_bits_equal(mv.cpu().numpy(), port.reduce(op[3:], x, 0), f"merged {op} value")
        return
    m = gpu.merge_partials(op, vals)
    gpu.sync()
    want = port.reduce(op, x, 0)
    if op == "sum" and dtype == np.float32:
        x64 = x.astype(np.float64)
        assert_sum_close(m.cpu().numpy(), want, np.abs(x64).sum(0), "merged sum", exact=x64.sum(0))
    else:
        assert_bits_equal(m.cpu().numpy(), want, f"merged {op}")


@pytest.mark.parametrize("dtype", [np.float32, np.int32], ids=["f32", "i32"])
def test_reduce_sharded_native_one_rank(gpu, port, dtype):
    """mtxc_reduce_sharded with a one-rank communicator (no NCCL involved): the local kernels, the
    gather-buffer slots and the merge must give the unsharded reduction; mtxc_allreduce is the identity;
    a gather buffer too small for the partials is refused with MTXC_ERR_WORKSPACE."""
    import torch

    from matrix_b200 import _abi
    from matrix_b200.shard import NativeComm, reduce_sharded

    rng = np.random.default_rng(9)
    shape = [37, 129, 33]
    if dtype == np.float32:
        x = (np.floor(rng.standard_normal(shape) * 4) / 4).astype(np.float32)
        x[4, 2, :] = np.nan
    else:
        x = make_values(rng, int(np.prod(shape)), dtype, "full").reshape(shape)
    xd = torch.from_numpy(x).cuda()
    with NativeComm() as comm:
        assert (comm.world, comm.rank) == (1, 0)
        for op in ("sum", "max", "min", "argmax", "argmin"):
            got = reduce_sharded(op, xd, 0, shape[0], comm=comm)
            gpu.sync()
            want = port.reduce(op, x, 0)
            if op == "sum" and dtype == np.float32:
                x64 = x.astype(np.float64)
                assert_sum_close(got.cpu().numpy(), want, np.abs(x64).sum(0), "native sum", exact=x64.sum(0))
            else:
                assert_bits_equal(got.cpu().numpy(), want, f"native {op}")
        buf = xd[0].clone().reshape(-1)
        gpu.allreduce("max", buf)
        gpu.sync()
        assert_bits_equal(buf.cpu().numpy(), x[0].reshape(-1), "one-rank allreduce")
    with NativeComm(buffer_bytes=256) as small:
        with pytest.raises(_abi.MtxcError) as e:
            reduce_sharded("sum", xd, 0, shape[0], comm=small)
        assert e.value.code == _abi.ERR_WORKSPACE


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_rank_run(extra_env):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=repo, **extra_env)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(repo, "tests", "multirank_shard_check.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    errs = [l for l in res.stderr.splitlines() if "Error" in l or "error" in l or "what()" in l][:20]
    assert res.returncode == 0, res.stdout[-3000:] + "\n".join(errs) + res.stderr[-2000:]
    assert res.stdout.count("rank ok") == 2, res.stdout[-2000:]
    return res.stdout


def test_reduce_sharded_on_two_gpus():
    """torchrun, 2 ranks on 2 GPUs: every op over the sharded and a local axis against the oracle, through
    the peer-memory exchange (one kernel over NVLink) -- skipped on 1 GPU."""
    out = _two_rank_run({})
    assert out.count("peer=1") == 2, out[-2000:]


def test_reduce_sharded_on_two_gpus_nccl_path():
    """The same with MTXC_COMM_PEER=0: the NCCL all-gather + merge kernel path."""
    out = _two_rank_run({"MTXC_COMM_PEER": "0"})
    assert out.count("peer=0") == 2, out[-2000:]


def test_peer_exchange_wait_is_bounded():
    """Rank 1 skips an exchange rank 0 makes: rank 0's wait runs out after MTXC_COMM_SPIN_LIMIT sleeps, the
    kernel returns and mtxc_comm_status reports it (no hang, no fault)."""
    out = _two_rank_run({"MTXC_SHARD_CHECK_TIMEOUT": "1", "MTXC_COMM_SPIN_LIMIT": "20000"})
    assert "timeout reported" in out, out[-2000:]
    # 20,000 polls of ~64 ns sleeps: milliseconds, far below the process group's 60 s timeout, so the kernel's
    # own bound ended the wait
    waited = float(re.search(r"rank 0 waited ([0-9.]+) s", out).group(1))
    assert waited < 10.0, out[-2000:]
