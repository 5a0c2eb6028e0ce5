"""Builds the CPU oracle (test infrastructure only).

* ``oracle/liboracle.so`` from ``oracle/oracle.cpp``: the restatement of the reference CPU eval.
* ``oracle/_ref/libmtx_ref.so`` via ``oracle/build_ref.py``: the reference's own CPU loops,
  built only where the reference tree is present.

Both are built for baseline x86-64 (no -march=native): they are built here and run on the GPU
box's host as well.  ``-ffp-contract=off`` keeps the float loops one rounding per operation.
"""
from __future__ import annotations

import importlib.util
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent

LIB = HERE / "liboracle.so"


def build_port() -> Path:
    src = HERE / "oracle.cpp"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["g++", "-std=c++17", "-O3", "-ffp-contract=off", "-fPIC", "-shared", "-pthread",
                        "-Wall", "-o", str(LIB), str(src)], check=True)
    return LIB


def build(quiet: bool = True) -> None:
    build_port()
    spec = importlib.util.spec_from_file_location("oracle_build_ref", HERE / "build_ref.py")
    build_ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build_ref)
    build_ref.build(build_ref.reference_root(None), quiet=quiet)


if __name__ == "__main__":
    build(quiet=False)
