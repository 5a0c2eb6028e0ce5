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
