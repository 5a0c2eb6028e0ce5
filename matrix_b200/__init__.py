"""matrix_b200: a B200 (sm_100a) backend for the reduce / broadcast hot path of AlanAditya/matrix.

The product is the C-ABI library ``matrix_b200/lib/libmtxc.so`` (include/mtxc.h).  This package
holds its build recipe (``build.py``), its ctypes binding (``_abi.py``) and a Python driver that
mirrors the reference's frontends on device tensors (``backend.py``).
"""
from ._abi import LIB_PATH, MtxcError, lib  # noqa: F401

__all__ = ["LIB_PATH", "MtxcError", "lib"]
