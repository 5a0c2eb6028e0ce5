"""Builds libmtxc.so (the C-ABI backend) in-tree for sm_100a.

Run as ``python -m matrix_b200.build`` (or through ``__graft_entry__.build()``).  nvcc
cross-compiles without a GPU.  Objects go to ``matrix_b200/_build/``; the library to
``matrix_b200/lib/libmtxc.so``, which travels with the source tree to the GPU box.  The
CUDA runtime is linked statically so the library does not depend on which libcudart the
host process (e.g. PyTorch) loaded.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmtxc.so"
HOST = PKG / "host"
HOST_LIB = LIBDIR / "libmtx.so"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    jobs = []
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]) or ptxas_info:
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd[1:1] = ["-Xptxas", "-v"]
            jobs.append(cmd)
    for src in sorted(CSRC.glob("*.cpp")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            jobs.append(["g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj)])

    def run(cmd: list[str]) -> str:
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        return res.stdout + res.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for out in ex.map(run, jobs):
            if out.strip() and (verbose or ptxas_info):
                print(out, file=sys.stderr)
    if jobs or not LIB.exists() or _stale(LIB, objs):
        run([nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs), "-ldl"])
    # the C++ host mirror of the reference API (mtx.hpp), a plain C++ library over the C ABI
    host_srcs = sorted(HOST.glob("*.cpp"))
    if host_srcs and (not HOST_LIB.exists() or _stale(HOST_LIB, [*host_srcs, *HOST.glob("*.hpp"), LIB, *headers])):
        cuda_include = Path(nvcc()).resolve().parent.parent / "include"  # NVTX v3 (header-only)
        run(["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", "-shared", "-I", str(INCLUDE), "-I", str(HOST),
             "-I", str(cuda_include), "-o", str(HOST_LIB), *map(str, host_srcs), "-L", str(LIBDIR), "-lmtxc",
             "-ldl", "-Wl,-rpath,$ORIGIN"])
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas-info" in sys.argv)
    print(LIB)
