"""ctypes binding of include/mtxc.h (libmtxc.so).

This is the binding a Python caller of the C ABI needs; it loads the in-tree library built by
``matrix_b200/build.py`` and fails loudly when it is missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmtxc.so"

MAX_DIMS = 8
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED_DTYPE = 2
ERR_SHAPE = 3
ERR_CUDA = 4
ERR_TIMEOUT = 5
ERR_NOT_INITIALIZED = 6
ERR_WORKSPACE = 7
ERR_COMM = 8
COMM_ID_BYTES = 128

REDUCE_OPS = {"sum": 0, "max": 1, "min": 2, "argmax": 3, "argmin": 4}
BINARY_OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "max": 4, "min": 5, "equal": 6}
UNARY_OPS = {"exp": 0, "sqrt": 1}
STATS = {"mean": 0, "rms": 1, "norm": 2}
POINTWISE_OPS = {"greater": 0, "less": 1, "logical_and": 2, "where": 3, "floor": 4, "full": 5, "arctan2": 6,
                 "arcsin": 7}


class MtxcError(RuntimeError):
    """A non-zero status from the C ABI, with mtxc_last_error()'s message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"mtxc error {code}: {message}")
        self.code = code


U32P = C.POINTER(C.c_uint32)
_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} not found: build it with `python -m matrix_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        i32, u32, u64, sz, vp = C.c_int, C.c_uint32, C.c_uint64, C.c_size_t, C.c_void_p
        sigs = {
            "mtxc_abi_version": (i32, []),
            "mtxc_init": (i32, [i32]),
            "mtxc_shutdown": (i32, []),
            "mtxc_last_error": (C.c_char_p, []),
            "mtxc_device_count": (i32, [C.POINTER(i32)]),
            "mtxc_set_stream": (i32, [vp]),
            "mtxc_use_own_stream": (i32, []),
            "mtxc_get_stream": (vp, []),
            "mtxc_sync": (i32, []),
            "mtxc_set_workspace": (i32, [vp, sz]),
            "mtxc_workspace_size": (i32, [C.POINTER(sz)]),
            "mtxc_reduce_workspace_bytes": (i32, [i32, i32, u32, u32, u32, U32P, U32P, U32P, C.POINTER(sz)]),
            "mtxc_alloc": (i32, [sz, C.POINTER(vp)]),
            "mtxc_free": (i32, [vp]),
            "mtxc_host_alloc": (i32, [sz, C.POINTER(vp)]),
            "mtxc_host_free": (i32, [vp]),
            "mtxc_upload": (i32, [vp, vp, sz]),
            "mtxc_download": (i32, [vp, vp, sz]),
            "mtxc_copy_device": (i32, [vp, vp, sz]),
            "mtxc_memset": (i32, [vp, i32, sz]),
            "mtxc_collapse_dims1": (u32, [U32P, U32P, u32, u64, U32P, U32P]),
            "mtxc_collapse_dims2": (u32, [U32P, U32P, U32P, u32, u64, U32P, U32P, U32P]),
            "mtxc_collapse_dims3": (u32, [U32P, U32P, U32P, U32P, u32, u64, U32P, U32P, U32P, U32P]),
            "mtxc_collapse_dims_reduce1": (u32, [U32P, U32P, u32, i32, i32, u64, U32P, U32P]),
            "mtxc_collapse_dims_reduce2": (u32, [U32P, U32P, U32P, u32, i32, i32, i32, u64, U32P, U32P, U32P]),
            "mtxc_collapse_dims_reduce3": (u32, [U32P, U32P, U32P, U32P, u32, i32, i32, u64, U32P, U32P, U32P, U32P]),
            "mtxc_broadcast_shapes": (i32, [U32P, U32P, i32, U32P, U32P, i32, U32P, U32P, U32P, U32P, U32P, U32P]),
            "mtxc_promote_types": (i32, [i32, i32]),
            "mtxc_reduce": (i32, [i32, i32, vp, vp, u32, u32, u32, U32P, U32P, U32P]),
            "mtxc_reduce_noalloc": (i32, [i32, i32, vp, vp, u32, u32, u32, U32P, U32P, U32P]),
            "mtxc_reduce_pair": (i32, [i32, i32, vp, vp, vp, u32, u32, u32, U32P, U32P, U32P]),
            "mtxc_merge_partials": (i32, [i32, i32, vp, vp, vp, vp, vp, u32, u64]),
            "mtxc_broadcast_binary": (i32, [i32, i32, vp, vp, vp, u32, U32P, U32P, U32P, U32P]),
            "mtxc_broadcast_binary_mixed": (i32, [i32, i32, i32, i32, vp, vp, vp, u32, U32P, U32P, U32P, U32P]),
            "mtxc_unary": (i32, [i32, i32, vp, vp, u32, U32P, U32P, U32P]),
            "mtxc_softmax_lastdim": (i32, [i32, vp, vp, u64, u32, u64, u64]),
            "mtxc_astype": (i32, [i32, i32, vp, vp, u32, U32P, U32P, U32P]),
            "mtxc_reduce_stat": (i32, [i32, i32, vp, vp, u32, u32, u32, U32P, U32P, U32P]),
            "mtxc_reduce_stat_dtype": (i32, [i32, i32, u32]),
            "mtxc_pointwise_collapse": (u32, [U32P, u32, U32P, u32, U32P, U32P]),
            "mtxc_pointwise": (i32, [i32, i32, vp, C.POINTER(vp), u32, u32, U32P, U32P]),
            "mtxc_comm_unique_id": (i32, [vp, sz]),
            "mtxc_comm_init": (i32, [i32, i32, vp, sz]),
            "mtxc_comm_destroy": (i32, []),
            "mtxc_comm_size": (i32, [C.POINTER(i32), C.POINTER(i32)]),
            "mtxc_comm_status": (i32, [C.POINTER(i32), C.POINTER(i32)]),
            "mtxc_reduce_sharded": (i32, [i32, i32, vp, vp, u32, u32, u32, U32P, U32P, U32P, C.POINTER(C.c_int64)]),
            "mtxc_allreduce": (i32, [i32, i32, vp, u64]),
            "mtxc_arange": (i32, [i32, vp, vp, vp, u64]),
            "mtxc_graph_begin": (i32, []),
            "mtxc_graph_end": (i32, [C.POINTER(vp)]),
            "mtxc_graph_launch": (i32, [vp]),
            "mtxc_graph_destroy": (i32, [vp]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        msg = lib().mtxc_last_error()
        raise MtxcError(rc, msg.decode() if msg else "")


def u32_array(values, n: int = MAX_DIMS):
    a = (C.c_uint32 * n)()
    for i, v in enumerate(values):
        v = int(v)
        if v < 0 or v > 0xFFFFFFFF:
            raise ValueError(f"value {v} does not fit the reference's 32-bit size_m")
        a[i] = v
    return a
