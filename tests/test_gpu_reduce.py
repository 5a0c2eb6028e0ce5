"""GPU parity of the axis reductions against the CPU oracle (the reference's CPU eval).

Each case states the op the way the reference's user writes it, ``x.<op>(axis, keepdims)``,
runs it through mtxc_reduce (via matrix_b200.backend, which derives the collapsed metadata
with the library's own collapse_dims_reduce), and compares with the oracle's evaluation of the
same op on the same bytes.  Rules: see tests/helpers.py.
"""
import zlib

import numpy as np
import pytest

from tests.helpers import (INT_DTYPES, assert_bits_equal, assert_sum_close, device_view, make_values,
                           strided_view, to_device)

pytestmark = pytest.mark.gpu

OPS = ["sum", "max", "min", "argmax", "argmin"]


def check_reduce(backend, port, op, base, shape, strides, offset, axis, keepdims, what="", dbase=None):
    x = strided_view(base, shape, strides, offset)
    cpu = port.reduce(op, x, axis, keepdims)
    if dbase is None:
        dbase = to_device(base)
    xd = device_view(dbase, shape, strides, offset)
    out = backend.reduce(op, xd, axis, keepdims)
    backend.sync()
    gpu = out.cpu().numpy()
    tag = f"{what} {op} shape={shape} strides={strides} off={offset} axis={axis} keep={keepdims} {base.dtype}"
    if op == "sum" and base.dtype == np.float32:
        x64 = x.astype(np.float64)
        abs_sum = np.sum(np.abs(x64), axis=axis, keepdims=keepdims)
        assert_sum_close(gpu, cpu, abs_sum, tag, exact=np.sum(x64, axis=axis, keepdims=keepdims))
    else:
        assert_bits_equal(gpu, cpu, tag)


def contiguous_case(rng, shape, dtype, kind="normal", extremes=True):
    n = int(np.prod(shape))
    base = make_values(rng, max(n, 1), dtype, kind, extremes)
    strides = [int(np.prod(shape[i + 1:])) for i in range(len(shape))]
    return base, strides


SHAPES = [
    [7], [1], [1000], [5, 3], [3, 5, 7], [2, 3, 4, 5], [2, 1, 3, 1, 4], [33, 1000], [4, 100003], [3, 1 << 20],
    [8, 513, 129], [16, 300, 64], [2, 3, 4, 5, 6, 7], [1, 1, 4096], [4096, 2], [2, 4096], [65, 31, 33],
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("op", OPS)
def test_reduce_shapes_f32(gpu, port, shape, op):
    rng = np.random.default_rng(zlib.crc32(f"{op}{shape}".encode()))
    base, strides = contiguous_case(rng, shape, np.float32, "ties" if op != "sum" else "normal")
    for axis in range(-len(shape), len(shape)):
        for keep in (False, True):
            check_reduce(gpu, port, op, base, shape, strides, 0, axis, keep)


@pytest.mark.parametrize("dtype", INT_DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("op", OPS)
def test_reduce_int_dtypes(gpu, port, dtype, op):
    rng = np.random.default_rng(11)
    for shape in ([3, 5, 7], [17, 2049], [8, 513, 129], [5, 100003], [2, 1 << 18]):
        base, strides = contiguous_case(rng, shape, dtype, "full")  # full range: sums wrap
        for axis in range(len(shape)):
            check_reduce(gpu, port, op, base, shape, strides, 0, axis, False)


NARROW = [np.int8, np.uint8, np.int16, np.uint16, np.bool_]


def narrow_pattern(rng, kind, shape, axis, dtype):
    """Values along `axis` of `shape` that steer the packed column extremum through each branch:
    random over the full range, heavy ties (four distinct values), rising or falling along the
    reduced axis (a new best every row), constant, and all at the type's lowest or highest value
    (no row ever beats the initial state)."""
    dt = np.dtype(dtype)
    lo, hi = (0, 1) if dt == np.bool_ else (np.iinfo(dt).min, np.iinfo(dt).max)
    n = int(np.prod(shape))
    if kind == "random":
        v = rng.integers(lo, hi + 1, n, dtype=np.int64)
    elif kind == "ties":
        v = rng.integers(lo, lo + 4 if dt != np.bool_ else 2, n, dtype=np.int64)
    elif kind in ("rising", "falling"):
        pos = np.indices(shape)[axis].reshape(-1).astype(np.int64)
        span = hi - lo
        step = pos * span // max(shape[axis] - 1, 1)
        v = lo + step if kind == "rising" else hi - step
    elif kind == "constant":
        v = np.full(n, lo + (hi - lo) // 3, dtype=np.int64)
    else:  # "low" / "high"
        v = np.full(n, lo if kind == "low" else hi, dtype=np.int64)
    return v.astype(dt)


@pytest.mark.parametrize("dtype", NARROW, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("op", ["max", "min", "argmax", "argmin"])
def test_reduce_narrow_packed(gpu, port, dtype, op):
    """Max / Min / ArgMax / ArgMin of the 1- and 2-byte types through the packed folds: over a strided
    axis, the 16-byte lanes (inner extent a multiple of 16 bytes), the 4-byte fallback lanes (a multiple
    of 4 bytes, or an operand offset that breaks 16-byte alignment) and the split path (long reduced
    axis); over rows, lanes along the row.  Each with value patterns that make every row (or vector) win
    some lane or none, and with chunks of 1, 3 and 7 rows besides the default, so the 16-bit chunk
    numbers turn into indices mid-run.  Bit-exact, first index of a tie."""
    rng = np.random.default_rng(zlib.crc32(f"narrow{op}{np.dtype(dtype).name}".encode()))
    code = 7 if dtype == np.bool_ else None
    cases = [([300, 64], 0, 0), ([3, 257, 48], 1, 0), ([1000, 20], 0, 0), ([700, 96], 0, 4), ([20000, 32], 0, 0),
             # rows: the same packed fold with the lanes along the row (warp and CTA per row, a split row,
             # an odd length, a start off the 16-byte boundary)
             ([64, 3000], 1, 0), ([8, 70001], 1, 0), ([5, 4099], 1, 3)]
    set_chunk = _col_chunk_setter()
    # the default chunk (65,535 rows: one chunk per lane at these sizes), then chunks of 1, 3 and 7 rows,
    # which turn the 16-bit chunk row numbers into indices at every row or in the middle of the lane's rows
    for chunk in (65535, 1, 3, 7):
        set_chunk(chunk)
        try:
            for shape, axis, off in (cases if chunk == 65535 else cases[:2] + cases[5:]):
                strides = [int(np.prod(shape[i + 1:])) for i in range(len(shape))]
                for kind in ("random", "ties", "rising", "falling", "constant", "low", "high"):
                    v = narrow_pattern(rng, kind, shape, axis, dtype)
                    base = np.concatenate([np.zeros(off, dtype=v.dtype), v])
                    x = strided_view(base, shape, strides, off)
                    cpu = port.reduce(op, x, axis, False, dtype_code=code) if code else port.reduce(op, x, axis, False)
                    out = gpu.reduce(op, device_view(to_device(base), shape, strides, off), axis)
                    gpu.sync()
                    assert_bits_equal(out.cpu().numpy(), cpu,
                                      f"{np.dtype(dtype).name} {op} {shape} axis {axis} +{off} {kind} chunk {chunk}")
        finally:
            set_chunk(65535)


def _col_chunk_setter():
    import ctypes

    from matrix_b200 import _abi

    fn = _abi.lib().mtxc_debug_set_col_chunk
    fn.argtypes, fn.restype = [ctypes.c_uint32], ctypes.c_uint32
    return fn


@pytest.mark.parametrize("op", OPS)
def test_reduce_float_specials(gpu, port, op):
    """NaN never wins, the first of equal extremes (incl. -0.0 / +0.0) is kept, rows of only
    NaN / -inf / lowest give the initial value and index 0."""
    rng = np.random.default_rng(5)
    for shape in ([64, 257], [33, 1000], [4, 70000], [300, 9, 40], [3, 1 << 17]):
        # no +-FLT_MAX in sums: where fp32 partial sums overflow, a sequential and a tree sum
        # may legitimately end in +inf vs NaN
        base, strides = contiguous_case(rng, shape, np.float32, "special", extremes=(op != "sum"))
        for axis in range(len(shape)):
            check_reduce(gpu, port, op, base, shape, strides, 0, axis, False)
    lowest = -np.finfo(np.float32).max
    rows = np.array([
        [np.nan] * 40,
        [-np.inf] * 40,
        [lowest] * 40,
        [-np.inf] * 20 + [lowest] + [-np.inf] * 19,
        [0.0, -0.0] * 20,
        [-0.0, 0.0] * 20,
        [np.nan, -0.0, 0.0] + [-1.0] * 37,
        [np.inf] * 40,
        [-np.inf, np.nan] * 20,
    ], dtype=np.float32)
    base = rows.reshape(-1)
    check_reduce(gpu, port, op, base, list(rows.shape), [40, 1], 0, 1, False, "special rows")
    check_reduce(gpu, port, op, base, list(rows.shape), [40, 1], 0, 0, False, "special cols")
    # the same runs long enough for the vector body and split partials
    long_rows = np.repeat(rows, 2000, axis=1)
    check_reduce(gpu, port, op, long_rows.reshape(-1), list(long_rows.shape), [80000, 1], 0, 1, False, "long special")


@pytest.mark.parametrize("op", OPS)
def test_reduce_strided_views(gpu, port, op):
    """Non-contiguous inputs: transposes, slices with offsets (unaligned starts), stride-0
    (expanded) axes."""
    rng = np.random.default_rng(7)
    base = make_values(rng, 1 << 20, np.float32, "ties")
    cases = [
        ([64, 100], [1, 128], 0),           # transposed
        ([16, 40, 30], [1200, 1, 40], 3),   # inner axes swapped, odd offset
        ([50, 1000], [1024, 1], 1),         # row slice, unaligned start
        ([50, 1000], [1024, 1], 5),
        ([7, 9, 300], [3000, 300, 1], 2),
        ([8, 16, 64], [0, 64, 1], 0),       # expanded leading axis
        ([8, 16, 64], [1024, 0, 1], 4),     # expanded middle axis
        ([100, 33], [40, 1], 3),
        ([10, 20, 30], [1, 10, 200], 1),    # fully transposed
        ([6, 5000], [2, 12], 0),
    ]
    for shape, strides, off in cases:
        for axis in range(len(shape)):
            for keep in (False, True):
                check_reduce(gpu, port, op, base, shape, strides, off, axis, keep)


def test_reduce_empty_and_degenerate(gpu, port):
    rng = np.random.default_rng(3)
    base = make_values(rng, 64, np.float32)
    for op in OPS:
        # zero-length reduced axis: outputs are the initial values (0, lowest, max, index 0)
        check_reduce(gpu, port, op, base, [4, 0], [1, 1], 0, 1, False, "len0")
        check_reduce(gpu, port, op, base, [3, 0, 5], [5, 5, 1], 0, 1, False, "len0 mid")
        # a single element
        check_reduce(gpu, port, op, base, [1], [1], 0, 0, False, "single")
        # full reduction of a vector: cdims == 0 (one output)
        check_reduce(gpu, port, op, base, [64], [1], 0, 0, False, "vector")
    # empty output: nothing is written and nothing faults
    import torch

    x = torch.empty((0, 5), device="cuda", dtype=torch.float32)
    out = gpu.reduce("sum", x, 1)
    gpu.sync()
    assert out.shape == (0,)


def test_reduce_int32_wraps(gpu, port):
    """int32 sums wrap exactly like the reference's int accumulator."""
    n = 1 << 16
    base = np.full(n * 4, 2**30 + 7, dtype=np.int32)
    base[1::3] = -(2**31)
    check_reduce(gpu, port, "sum", base, [4, n], [n, 1], 0, 1, False, "wrap rows")
    check_reduce(gpu, port, "sum", base, [4, n], [n, 1], 0, 0, False, "wrap cols")


def test_reduce_split_workspace_too_small(gpu, port):
    """With no workspace the split count drops to 1 and results are unchanged."""
    from matrix_b200 import _abi

    rng = np.random.default_rng(9)
    base = make_values(rng, 8 * (1 << 20), np.float32, "ties")
    L = _abi.lib()
    import ctypes

    size = ctypes.c_size_t()
    _abi.check(L.mtxc_workspace_size(ctypes.byref(size)))
    import torch

    keep = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    try:
        _abi.check(L.mtxc_set_workspace(None, 0))
        for op in OPS:
            check_reduce(gpu, port, op, base, [8, 1 << 20], [1 << 20, 1], 0, 1, False, "no workspace")
    finally:
        _abi.check(L.mtxc_set_workspace(keep.data_ptr(), size.value))
    # keep the replacement workspace alive for the rest of the session
    test_reduce_split_workspace_too_small.workspace = keep


@pytest.mark.parametrize("dtype", [np.int8, np.uint8, np.bool_], ids=lambda d: np.dtype(d).name)
def test_reduce_narrow_column_sums(gpu, port, dtype):
    """Sum (and the fused uint8 / int8 mean) of the 1-byte types over a strided axis, through the column
    kernel's 16-bit-lane fold: long columns with the default workspace and with none (one split, so each
    thread folds ~375 rows and the lanes are masked back to their low byte mid-run), 16-byte aligned
    operands and one 4 bytes off the boundary (the 4-byte lanes).  Full-range values: the sums wrap.
    Bit-exact."""
    import ctypes

    import torch

    from matrix_b200 import _abi

    rng = np.random.default_rng(zlib.crc32(f"colsum{np.dtype(dtype).name}".encode()))
    L = _abi.lib()
    size = ctypes.c_size_t()
    _abi.check(L.mtxc_workspace_size(ctypes.byref(size)))
    keep = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    cases = [([3000, 512], 0, 0), ([2, 2100, 64], 1, 0), ([1100, 96], 0, 4), ([5000, 16], 0, 16)]
    try:
        for ws in ("default", "none"):
            if ws == "none":
                _abi.check(L.mtxc_set_workspace(None, 0))
            for shape, axis, off in cases:
                n = int(np.prod(shape))
                v = rng.integers(0, 2, n).astype(np.bool_) if dtype == np.bool_ else make_values(rng, n, dtype, "full")
                base = np.concatenate([np.zeros(off, dtype=v.dtype), v])
                strides = [int(np.prod(shape[i + 1:])) for i in range(len(shape))]
                check_reduce(gpu, port, "sum", base, shape, strides, off, axis, False, f"workspace {ws}")
                if dtype != np.bool_:
                    x = strided_view(base, shape, strides, off)
                    want, _ = port.stat("mean", x, axis, False)
                    got = gpu.stat("mean", device_view(to_device(base), shape, strides, off), axis, False)
                    gpu.sync()
                    assert_bits_equal(got.cpu().numpy(), np.asarray(want),
                                      f"mean {np.dtype(dtype).name} {shape} axis {axis} +{off} workspace {ws}")
    finally:
        _abi.check(L.mtxc_set_workspace(keep.data_ptr(), size.value))
    test_reduce_narrow_column_sums.workspace = keep


def test_unsupported_dtype_is_an_error(gpu):
    import torch

    from matrix_b200 import _abi

    x = torch.zeros(16, dtype=torch.float32, device="cuda")
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    meta = gpu.reduce_meta([16], [1], 0)
    shape, so, si = meta.arrays
    rc = _abi.lib().mtxc_reduce(0, 9, out.data_ptr(), x.data_ptr(), 1, 16, meta.cdims, shape, so, si)  # Complex64
    assert rc == _abi.ERR_UNSUPPORTED_DTYPE
    assert b"Complex64" in _abi.lib().mtxc_last_error()
    rc = _abi.lib().mtxc_reduce(0, 13, out.data_ptr(), x.data_ptr(), 1, 16, meta.cdims, shape, so, si)
    assert rc == _abi.ERR_UNSUPPORTED_DTYPE
    rc = _abi.lib().mtxc_reduce(9, 0, out.data_ptr(), x.data_ptr(), 1, 16, meta.cdims, shape, so, si)
    assert rc == _abi.ERR_INVALID_ARGUMENT


# ------------------------------------------------------------------------------------------
# The benchmark configs at full size (C1, C3, C4) and C5b at reduced size
# ------------------------------------------------------------------------------------------
@pytest.mark.slow
def test_config1_sum_last_axis(gpu, port):
    rng = np.random.default_rng(0)
    base = rng.standard_normal(1024 * 4096).astype(np.float32)
    check_reduce(gpu, port, "sum", base, [1024, 4096], [4096, 1], 0, -1, False, "C1")


@pytest.mark.slow
def test_config3_max_argmax_axis1(gpu, port):
    """Max and ArgMax (and Min / ArgMin) along axis 1 of [64, 8192, 1024], values quantised to
    multiples of 1/256 so that every output has ties: indices must be the first ones."""
    rng = np.random.default_rng(2)
    n = 64 * 8192 * 1024
    base = (np.floor(rng.random(n, dtype=np.float32) * 256) / 256).astype(np.float32)
    dbase = to_device(base)
    for op in ("max", "argmax", "min", "argmin"):
        check_reduce(gpu, port, op, base, [64, 8192, 1024], [8192 * 1024, 1024, 1], 0, 1, False, "C3", dbase)


@pytest.mark.slow
@pytest.mark.parametrize("dtype", [np.float32, np.int32], ids=["f32", "i32"])
def test_config4_sum_axes_0_2(gpu, port, dtype):
    """Sum over axes (0, 2) of [32, 4096, 2048] as x.sum(2).sum(0), both steps on the GPU."""
    import torch

    rng = np.random.default_rng(3)
    shape = [32, 4096, 2048]
    n = int(np.prod(shape))
    if dtype == np.float32:
        base = rng.standard_normal(n).astype(np.float32)
    else:
        base = rng.integers(-1000, 1000, n, dtype=np.int32, endpoint=True)
    x = base.reshape(shape)
    cpu = port.reduce("sum", port.reduce("sum", x, 2), 0)
    xd = torch.from_numpy(base).cuda().reshape(shape)
    gpu_out = gpu.reduce("sum", gpu.reduce("sum", xd, 2), 0)
    gpu.sync()
    g = gpu_out.cpu().numpy()
    if dtype == np.int32:
        assert_bits_equal(g, cpu, "C4 i32")
    else:
        x64 = x.astype(np.float64)
        assert_sum_close(g, cpu, np.abs(x64).sum(axis=(0, 2)), "C4 f32", exact=x64.sum(axis=(0, 2)))


@pytest.mark.slow
def test_config5b_full_sum_reduced(gpu, port):
    """The full Sum of C5b on an [8, 2^26] view (2 GiB): sum(1) then sum(0)."""
    import torch

    rng = np.random.default_rng(4)
    shape = [8, 1 << 26]
    base = rng.standard_normal(shape[0] * shape[1], dtype=np.float32)
    x = base.reshape(shape)
    cpu = port.reduce("sum", port.reduce("sum", x, 1), 0)
    xd = torch.from_numpy(base).cuda().reshape(shape)
    g = gpu.reduce("sum", gpu.reduce("sum", xd, 1), 0)
    gpu.sync()
    b64 = base.astype(np.float64)
    assert_sum_close(g.cpu().numpy(), cpu, np.array(np.abs(b64).sum()), "C5b", exact=np.array(b64.sum()))
