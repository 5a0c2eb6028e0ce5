"""The C-ABI library without a GPU: it loads, exports every function include/mtxc.h declares,
and refuses device work on a thread that did not call mtxc_init."""
import ctypes as C
import re
import subprocess

from tests.conftest import REPO


def declared_functions():
    text = (REPO / "include" / "mtxc.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(mtxc_[a-z0-9_]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_hot_path():
    names = declared_functions()
    for must in ("mtxc_init", "mtxc_reduce", "mtxc_broadcast_binary", "mtxc_unary", "mtxc_collapse_dims_reduce2",
                 "mtxc_broadcast_shapes", "mtxc_sync", "mtxc_graph_begin", "mtxc_astype", "mtxc_pointwise",
                 "mtxc_pointwise_collapse"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from matrix_b200 import _abi

    lib = _abi.lib()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/mtxc.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (mtxc_[a-z0-9_]+)", out))
    assert set(declared_functions()) <= exported
    assert lib.mtxc_abi_version() == 1


def test_calls_before_init_fail_cleanly():
    from matrix_b200 import _abi

    lib = _abi.lib()
    arr = _abi.u32_array
    rc = lib.mtxc_reduce(0, 0, None, None, 1, 4, 1, arr([4]), arr([1]), arr([4]))
    assert rc == _abi.ERR_NOT_INITIALIZED
    assert b"mtxc_init" in lib.mtxc_last_error()
    assert lib.mtxc_broadcast_binary(0, 0, None, None, None, 1, arr([4]), arr([1]), arr([1]), arr([1])) == \
        _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_unary(0, 0, None, None, 1, arr([4]), arr([1]), arr([1])) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_astype(0, 3, None, None, 1, arr([4]), arr([1]), arr([1])) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_reduce_stat(0, 0, None, None, 1, 4, 1, arr([4]), arr([1]), arr([4])) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_broadcast_binary_mixed(0, 0, 0, 3, None, None, None, 1, arr([4]), arr([1]), arr([1]),
                                           arr([1])) == _abi.ERR_NOT_INITIALIZED
    ptrs = (C.c_void_p * 3)()
    assert lib.mtxc_pointwise(0, 0, None, ptrs, 2, 1, arr([4]), arr([], 24)) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_softmax_lastdim(0, None, None, 1, 4, 4, 4) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_sync() == _abi.ERR_NOT_INITIALIZED
    size = C.c_size_t(123)
    assert lib.mtxc_workspace_size(C.byref(size)) == 0 and size.value == 0


def test_workspace_query_is_host_only():
    """mtxc_reduce_workspace_bytes plans without a device: a single long row needs split
    partials, a wide matrix does not."""
    from matrix_b200 import _abi

    lib = _abi.lib()
    arr = _abi.u32_array
    b = C.c_size_t()
    # full Sum of one run of 2^29 floats (cdims == 0): split across CTAs
    assert lib.mtxc_reduce_workspace_bytes(0, 0, 1, 1 << 29, 0, None, None, None, C.byref(b)) == 0
    assert b.value > 0
    # [131072, 2048] row sums: one warp per row, no partials
    assert lib.mtxc_reduce_workspace_bytes(0, 0, 1, 2048, 1, arr([131072]), arr([1]), arr([2048]), C.byref(b)) == 0
    assert b.value == 0
    # Float16 (code 1) is evaluated; Complex64 (code 9) is refused like dispatch_type refuses it
    assert lib.mtxc_reduce_workspace_bytes(0, 1, 1, 2048, 1, arr([16]), arr([1]), arr([2048]), C.byref(b)) == 0
    assert lib.mtxc_reduce_workspace_bytes(0, 9, 1, 2048, 1, arr([16]), arr([1]), arr([2048]), C.byref(b)) == \
        _abi.ERR_UNSUPPORTED_DTYPE
