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
    # the multi-GPU entry points: no device bound, no communicator
    assert lib.mtxc_comm_init(2, 0, b"\0" * _abi.COMM_ID_BYTES, 0) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_reduce_sharded(0, 0, None, None, 1, 4, 1, arr([4]), arr([1]), arr([4]), None) == \
        _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_allreduce(0, 0, None, 4) == _abi.ERR_NOT_INITIALIZED
    n, r = C.c_int(-1), C.c_int(-1)
    assert lib.mtxc_comm_size(C.byref(n), C.byref(r)) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_comm_status(C.byref(n), C.byref(r)) == _abi.ERR_NOT_INITIALIZED
    assert lib.mtxc_comm_destroy() == 0
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


def test_noalloc_scratch_covers_the_planned_reductions():
    """The split plans stay far inside mtxc_reduce_noalloc's static scratch: no reduction of these large
    shapes (rows, columns, every op, 1- to 8-byte types, pair states included) asks for more partial bytes
    than MTXC_NOALLOC_SCRATCH_BYTES, so the allocation-free entry point's refusal is a guard, not a
    limit callers meet.  (Host-only: the workspace query plans without a device.)"""
    from matrix_b200 import _abi

    lib, arr = _abi.lib(), _abi.u32_array
    scratch = 4 << 20
    worst = 0
    b = C.c_size_t()
    for dtype in (0, 1, 2, 3, 7, 8, 10, 11):
        for op in range(5):
            # rows: few long rows, many short rows
            for rows, length in ((1, 1 << 31), (8, 1 << 29), (1000, 1 << 20), (9000, 4096), (1 << 20, 256)):
                assert lib.mtxc_reduce_workspace_bytes(op, dtype, 1, length, 1, arr([rows]), arr([1]),
                                                       arr([length]), C.byref(b)) == 0
                worst = max(worst, b.value)
            # columns: a strided reduced axis over [outer, length, inner]
            for outer, length, inner in ((1, 1 << 22, 512), (32, 65536, 512), (1, 1 << 19, 4096), (64, 8192, 1024)):
                assert lib.mtxc_reduce_workspace_bytes(op, dtype, inner, length, 2, arr([outer, inner]),
                                                       arr([inner, 1]), arr([length * inner, 1]), C.byref(b)) == 0
                worst = max(worst, b.value)
    assert 0 < worst <= scratch, worst


def test_column_chunk_hook_clamps():
    """mtxc_debug_set_col_chunk (a test hook outside the public header) sets the rows per chunk of the
    packed column (value, index) fold within 1 .. 65,535 and returns the previous value."""
    from matrix_b200 import _abi

    fn = _abi.lib().mtxc_debug_set_col_chunk
    fn.argtypes, fn.restype = [C.c_uint32], C.c_uint32
    assert fn(7) == 65535
    assert fn(0) == 7
    assert fn(1 << 20) == 1
    assert fn(65535) == 65535


def test_every_mixed_pair_has_a_fused_kernel_family():
    """mtxc_broadcast_binary_mixed serves every pair of two different dtypes (Complex64 aside) from two
    kernel families: the promoted dtype is one operand's (mixed.cu, any result dtype), or a third one
    (mixed3.cu, which instantiates only Float, Int16 and Int32 results).  The promotion table must keep
    the third dtypes inside that set, and the split is 40 + 26 of the 66 pairs."""
    from matrix_b200 import _abi

    lib = _abi.lib()
    codes = [0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12]
    own = third = 0
    for i, a in enumerate(codes):
        for b in codes[i + 1:]:
            d = lib.mtxc_promote_types(a, b)
            assert d == lib.mtxc_promote_types(b, a)
            if d in (a, b):
                own += 1
            else:
                assert d in (0, 4, 3), (a, b, d)  # Float, Int16, Int32
                third += 1
    assert (own, third) == (40, 26)


def test_comm_unique_id_needs_no_gpu():
    """mtxc_comm_unique_id loads NCCL at run time (no link-time dependency) and draws an id on the host;
    a buffer shorter than MTXC_COMM_ID_BYTES is refused."""
    from matrix_b200 import _abi

    lib = _abi.lib()
    short = C.create_string_buffer(16)
    assert lib.mtxc_comm_unique_id(short, 16) == _abi.ERR_INVALID_ARGUMENT
    ids = []
    for _ in range(2):
        buf = C.create_string_buffer(_abi.COMM_ID_BYTES)
        rc = lib.mtxc_comm_unique_id(buf, _abi.COMM_ID_BYTES)
        assert rc == 0, lib.mtxc_last_error()
        ids.append(buf.raw)
    assert ids[0] != ids[1] and any(ids[0])
    out = subprocess.run(["ldd", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    assert "nccl" not in out
