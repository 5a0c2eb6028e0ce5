"""The C++ host mirror (matrix_b200/host/mtx.hpp, libmtx.so) on the GPU.

tests/cpp/test_host_mirror.cpp builds lazy graphs with the reference's API names (operators, axis
reductions, exp, eval / compile / execute, views) and checks them against the CPU oracle; this test
compiles it against the in-tree libraries and runs it.
"""
import os
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent


def test_host_mirror_program(tmp_path):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = REPO / "matrix_b200" / "lib"
    oracle_dir = REPO / "oracle"
    exe = tmp_path / "test_host_mirror"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(REPO / "include"), "-I", str(REPO / "matrix_b200" / "host"),
                    str(REPO / "tests" / "cpp" / "test_host_mirror.cpp"), "-o", str(exe),
                    "-L", str(lib), "-lmtx", "-lmtxc", "-L", str(oracle_dir), "-loracle",
                    f"-Wl,-rpath,{lib}", f"-Wl,-rpath,{oracle_dir}"], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=dict(os.environ))
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "0 failures" in res.stdout


@pytest.mark.parametrize("path", ["peer", "nccl"])
def test_host_mirror_sharded_two_gpus(tmp_path, path):
    """mtx::Communicator and mtx::reduce_sharded from C++, two processes on two GPUs (skipped on one):
    tests/cpp/test_mirror_sharded.cpp checks every op over the sharded axis against the oracle's reduction
    of the whole tensor, and a compiled pass replayed with new leaf contents; through the peer exchange and,
    with MTXC_COMM_PEER=0, through the NCCL all-gather + merge."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lib = REPO / "matrix_b200" / "lib"
    oracle_dir = REPO / "oracle"
    exe = tmp_path / "test_mirror_sharded"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(REPO / "include"), "-I", str(REPO / "matrix_b200" / "host"),
                    str(REPO / "tests" / "cpp" / "test_mirror_sharded.cpp"), "-o", str(exe),
                    "-L", str(lib), "-lmtx", "-lmtxc", "-L", str(oracle_dir), "-loracle",
                    f"-Wl,-rpath,{lib}", f"-Wl,-rpath,{oracle_dir}"], check=True)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if path == "nccl":
        env["MTXC_COMM_PEER"] = "0"
    id_file = tmp_path / "comm.id"
    procs = [subprocess.Popen(["timeout", "-k", "10", "120", str(exe), str(r), "2", str(id_file)],
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=env) for r in range(2)]
    outs = [p.communicate(timeout=150)[0] for p in procs]
    for r, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r}:\n{out[-3000:]}"
        assert f"rank {r} peer={1 if path == 'peer' else 0}" in out, out[-2000:]
        assert f"rank {r}: " in out and " 0 failures" in out, out[-2000:]
