"""Pins the oracle (oracle/oracle.cpp) to the reference's own CPU code.

oracle/_ref/libmtx_ref.so is the reference's hot-path CPU loops and shape helpers, compiled
unchanged from the reference tree by oracle/build_ref.py.  Every function of the restatement
must agree with it bit for bit on random metadata and random tensors.  The same comparison is
made for the product library's host-side shape folding (libmtxc.so's mtxc_collapse_dims*,
mtxc_broadcast_shapes, mtxc_promote_types), which needs no GPU.
"""
import ctypes as C

import numpy as np
import pytest

from tests.helpers import make_values, strided_view

DTYPES = [np.float32, np.int32, np.uint32, np.int64, np.uint64, np.int16, np.uint16, np.int8, np.uint8, np.float16]


def rand_meta(rng, dims):
    """Random shapes and strides: mostly plausible tensors, sometimes arbitrary uint32 values
    (including products that overflow 32 bits, where the reference's size_m arithmetic wraps)."""
    shape = [int(v) for v in rng.integers(1, 6, dims)]
    if rng.random() < 0.3:
        shape = [int(v) for v in rng.choice([1, 2, 3, 65536, 1 << 20, 3000000000], dims)]
    strides = []
    for _ in range(3):
        kind = rng.integers(0, 4)
        if kind == 0:
            s, acc = [0] * dims, 1
            for i in range(dims - 1, -1, -1):
                s[i] = acc & 0xFFFFFFFF
                acc *= shape[i]
        elif kind == 1:
            s = [int(v) for v in rng.integers(0, 1 << 32, dims, dtype=np.uint64)]
        elif kind == 2:
            s = [int(v) * int(rng.integers(0, 2)) for v in rng.integers(1, 50, dims)]
        else:
            s, acc = [0] * dims, 1
            for i in range(dims - 1, -1, -1):
                s[i] = 0 if rng.random() < 0.3 else acc & 0xFFFFFFFF
                acc *= shape[i]
        strides.append(s)
    return shape, strides


def test_collapse_functions_match_reference(port, ref):
    rng = np.random.default_rng(0)
    for trial in range(3000):
        dims = int(rng.integers(0, 9))
        shape, (s0, s1, s2) = rand_meta(rng, dims)
        cap = int(rng.choice([0x7FFFFFFF, 0xFFFFFFFF, 1000, 16]))
        for strides in ([s0], [s0, s1], [s0, s1, s2]):
            assert port.collapse(shape, *strides, cap=cap) == ref.collapse(shape, *strides, cap=cap), (shape, strides, cap)
        if dims == 0:
            continue
        axis = int(rng.integers(0, dims))
        keep = bool(rng.integers(0, 2))
        outer = bool(rng.integers(0, 2))
        for strides in ([s0], [s0, s1], [s0, s1, s2]):
            kw = dict(axis=axis, keep=keep, cap=cap)
            if len(strides) == 2:
                kw["outer"] = outer
            assert port.collapse_reduce(shape, *strides, **kw) == ref.collapse_reduce(shape, *strides, **kw), \
                (shape, strides, kw)


def test_broadcast_shapes_and_promotion_match_reference(port, ref):
    rng = np.random.default_rng(1)
    for trial in range(3000):
        d1, d2 = int(rng.integers(0, 8)), int(rng.integers(0, 8))
        base = [int(v) for v in rng.integers(1, 5, max(d1, d2))]
        s1 = [v if rng.random() < 0.7 else 1 for v in base[len(base) - d1:]]
        s2 = [v if rng.random() < 0.7 else 1 for v in base[len(base) - d2:]]
        if rng.random() < 0.1 and d1:
            s1[0] = 7  # usually incompatible
        t1 = [int(v) for v in rng.integers(0, 100, d1)]
        t2 = [int(v) for v in rng.integers(0, 100, d2)]
        try:
            want = ref.broadcast_shapes(s1, t1, s2, t2)
        except ValueError:
            with pytest.raises(ValueError):
                port.broadcast_shapes(s1, t1, s2, t2)
            continue
        assert port.broadcast_shapes(s1, t1, s2, t2) == want, (s1, t1, s2, t2)
    for a in range(13):
        for b in range(13):
            assert port.promote(a, b) == ref.promote(a, b)


def random_view(rng, dtype, max_elems=4000):
    dims = int(rng.integers(1, 5))
    shape = [int(v) for v in rng.integers(1, 9, dims)]
    if rng.random() < 0.2:
        shape[int(rng.integers(0, dims))] = int(rng.integers(20, 200))
    perm = rng.permutation(dims) if rng.random() < 0.4 else np.arange(dims)
    full = [shape[i] for i in perm]
    strides_full, acc = [0] * dims, 1
    for i in range(dims - 1, -1, -1):
        strides_full[i] = acc
        acc *= full[i] + (1 if rng.random() < 0.2 else 0)  # sometimes padded rows
    strides = [0] * dims
    for k, i in enumerate(perm):
        strides[i] = strides_full[k]
    if rng.random() < 0.2:
        strides[int(rng.integers(0, dims))] = 0  # an expanded axis
    off = int(rng.integers(0, 4))
    need = off + sum((e - 1) * s for e, s in zip(shape, strides)) + 1
    base = make_values(rng, need, dtype, "special" if np.dtype(dtype) == np.float32 else "full") \
        if np.dtype(dtype) != np.float16 else rng.standard_normal(need).astype(np.float16)
    return base, shape, strides, off


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
def test_reduce_loops_match_reference(port, ref, dtype):
    rng = np.random.default_rng(2)
    for trial in range(150):
        base, shape, strides, off = random_view(rng, dtype)
        x = strided_view(base, shape, strides, off)
        axis = int(rng.integers(0, len(shape)))
        keep = bool(rng.integers(0, 2))
        for op in ("sum", "max", "min", "argmax", "argmin"):
            a = port.reduce(op, x, axis, keep)
            b = ref.reduce(op, x, axis, keep)
            assert a.shape == b.shape and a.tobytes() == b.tobytes(), (op, shape, strides, off, axis, keep)


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: np.dtype(d).name)
def test_broadcast_loops_match_reference(port, ref, dtype):
    rng = np.random.default_rng(3)
    for trial in range(150):
        dims = int(rng.integers(1, 5))
        out = [int(v) for v in rng.integers(1, 7, dims)]
        sa = [v if rng.random() < 0.6 else 1 for v in out][int(rng.integers(0, dims)):]
        sb = [v if rng.random() < 0.6 else 1 for v in out]
        if not sa:
            sa = [1]
        a = make_values(rng, int(np.prod(sa)), dtype, "full") if np.dtype(dtype).kind in "iu" else \
            rng.standard_normal(int(np.prod(sa))).astype(dtype)
        b = make_values(rng, int(np.prod(sb)), dtype, "full") if np.dtype(dtype).kind in "iu" else \
            rng.standard_normal(int(np.prod(sb))).astype(dtype)
        a, b = a.reshape(sa), b.reshape(sb)
        for op in ("add", "sub", "mul", "div", "max", "min"):
            bb = b
            if op == "div" and np.dtype(dtype).kind in "iu":
                bb = b.copy()
                bb[bb == 0] = 1
                if np.dtype(dtype).kind == "i":
                    bb[bb == -1] = 3
            x = port.binary(op, a, bb)
            y = ref.binary(op, a, bb)
            assert x.shape == y.shape and x.tobytes() == y.tobytes(), (op, sa, sb)


def _bf16_bits(rng, n):
    """Random bfloat16 values as uint16 bits: normals with ties, and NaN, +-inf, +-0."""
    v = (np.floor(rng.standard_normal(n) * 8) / 8).astype(np.float32)
    pick = rng.integers(0, 16, n)
    v[pick == 0], v[pick == 1], v[pick == 2], v[pick == 3] = np.nan, np.inf, -np.inf, -0.0
    return (v.view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("kind", ["bool", "bfloat16"])
def test_bool_and_bfloat16_loops_match_reference(port, ref, kind):
    """Bool (code 7) and BFloat16 (code 10, carried as uint16 bits) through the same loops."""
    rng = np.random.default_rng(7)
    code = 7 if kind == "bool" else 10

    def values(n):
        return rng.integers(0, 2, n).astype(np.bool_) if kind == "bool" else _bf16_bits(rng, n)

    for trial in range(120):
        _, shape, strides, off = random_view(rng, np.float32)
        need = off + sum((e - 1) * s for e, s in zip(shape, strides)) + 1
        x = strided_view(values(need), shape, strides, off)
        axis = int(rng.integers(0, len(shape)))
        for op in ("sum", "max", "min", "argmax", "argmin"):
            a = port.reduce(op, x, axis, dtype_code=code)
            b = ref.reduce(op, x, axis, dtype_code=code)
            assert a.shape == b.shape and a.tobytes() == b.tobytes(), (kind, op, shape, strides, off, axis)
        sa = [int(v) for v in rng.integers(1, 6, 3)]
        sb = [sa[0], 1, sa[2]] if rng.random() < 0.5 else [1, sa[1], 1]
        a, b = values(int(np.prod(sa))).reshape(sa), values(int(np.prod(sb))).reshape(sb)
        for op in ("add", "sub", "mul", "div", "max", "min"):
            bb = np.ones_like(b) if (kind == "bool" and op == "div") else b  # bool / false traps on x86
            x1 = port.binary(op, a, bb, dtype_code=code)
            y1 = ref.binary(op, a, bb, dtype_code=code)
            assert x1.shape == y1.shape and x1.tobytes() == y1.tobytes(), (kind, op, sa, sb)


def test_exp_loop_matches_reference(port, ref):
    rng = np.random.default_rng(4)
    for trial in range(100):
        base, shape, strides, off = random_view(rng, np.float32)
        x = strided_view(base, shape, strides, off)
        assert port.exp(x).tobytes() == ref.exp(x).tobytes(), (shape, strides, off)


# ------------------------------------------------------------------------------------------
# The product's host-side shape folding (no GPU needed)
# ------------------------------------------------------------------------------------------
def _mtxc():
    from matrix_b200 import _abi

    return _abi.lib(), _abi.u32_array


def test_product_shape_folding_matches_oracle(port):
    L, arr = _mtxc()
    rng = np.random.default_rng(5)
    for trial in range(3000):
        dims = int(rng.integers(0, 9))
        shape, (s0, s1, s2) = rand_meta(rng, dims)
        cap = int(rng.choice([0x7FFFFFFF, 0xFFFFFFFF, 1000]))
        for strides in ([s0], [s0, s1], [s0, s1, s2]):
            n = len(strides)
            o = [arr([]) for _ in range(n + 1)]
            k = getattr(L, f"mtxc_collapse_dims{n}")(arr(shape), *[arr(s) for s in strides], dims, cap, *o)
            assert (k, [list(v[:k]) for v in o]) == port.collapse(shape, *strides, cap=cap)
        if not dims:
            continue
        axis, keep, outer = int(rng.integers(0, dims)), int(rng.integers(0, 2)), int(rng.integers(0, 2))
        for strides in ([s0], [s0, s1], [s0, s1, s2]):
            n = len(strides)
            o = [arr([]) for _ in range(n + 1)]
            extra = [outer] if n == 2 else []
            k = getattr(L, f"mtxc_collapse_dims_reduce{n}")(arr(shape), *[arr(s) for s in strides], dims, axis, keep,
                                                           *extra, cap, *o)
            kw = dict(axis=axis, keep=bool(keep), cap=cap)
            if n == 2:
                kw["outer"] = bool(outer)
            assert (k, [list(v[:k]) for v in o]) == port.collapse_reduce(shape, *strides, **kw)


def test_product_broadcast_shapes_and_promotion_match_oracle(port):
    L, arr = _mtxc()
    rng = np.random.default_rng(6)
    for trial in range(2000):
        d1, d2 = int(rng.integers(0, 8)), int(rng.integers(0, 8))
        base = [int(v) for v in rng.integers(1, 5, max(d1, d2))]
        s1 = [v if rng.random() < 0.7 else 1 for v in base[len(base) - d1:]]
        s2 = [v if rng.random() < 0.7 else 1 for v in base[len(base) - d2:]]
        if rng.random() < 0.1 and d1:
            s1[0] = 7
        t1 = [int(v) for v in rng.integers(0, 100, d1)]
        t2 = [int(v) for v in rng.integers(0, 100, d2)]
        outs = [arr([]) for _ in range(6)]
        rc = L.mtxc_broadcast_shapes(arr(s1), arr(t1), d1, arr(s2), arr(t2), d2, *outs)
        try:
            want = port.broadcast_shapes(s1, t1, s2, t2)
        except ValueError:
            assert rc == 3  # MTXC_ERR_SHAPE
            continue
        od = max(d1, d2)
        assert rc == 0 and [list(v[:od]) for v in outs] == want
    for a in range(13):
        for b in range(13):
            assert L.mtxc_promote_types(a, b) == port.promote(a, b)
    assert L.mtxc_promote_types(13, 0) == -1


@pytest.mark.parametrize("dtype", [np.float32, np.int32, np.float16, np.uint8])
def test_flat_sum_matches_reference_loop(port, ref, dtype):
    """The restatement's full Sum with a 64-bit count (config 5b's 2^32 elements exceed size_m) equals the
    reference's own Sum loop, run as x.flatten().sum(0), bit for bit wherever the latter can count."""
    rng = np.random.default_rng(12)
    for n in (0, 1, 7, 4096, 1 << 20, 3_000_001):
        if dtype == np.float32:
            x = rng.standard_normal(n).astype(np.float32)
        elif dtype == np.float16:
            x = rng.standard_normal(n).astype(np.float16)
        else:
            info = np.iinfo(dtype)
            x = rng.integers(info.min, info.max, n, dtype=np.int64).astype(dtype)
        want = ref.reduce("sum", x, 0) if n else np.zeros((), dtype=dtype)
        got = port.sum_flat(x)
        assert np.asarray(got).tobytes() == np.asarray(want, dtype=dtype).reshape(()).tobytes(), (n, got, want)
