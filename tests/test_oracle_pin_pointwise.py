"""Pins the oracle's astype, exp / sqrt, equal and make_pointwise restatements (oracle/oracle.cpp)
to the reference's own CPU code in oracle/_ref/libmtx_ref.so (copyCPUinplaceTypeCasted, the sqrt and
exp lambdas, equal_backend's loop, make_pointwise's collapse and the greater / less / logical_and /
where / floor / full backends, compiled unchanged by oracle/build_ref.py), bit for bit.  The product
library's own mtxc_pointwise_collapse is checked against the oracle the same way (host code, no GPU).
"""
import ctypes as C

import numpy as np
import pytest


NUMPY_TYPES = [np.float32, np.float16, np.uint8, np.int32, np.int16, np.uint32, np.uint16, np.bool_, np.int8,
               np.int64, np.uint64]
CODES = {np.dtype(t): c for t, c in zip(NUMPY_TYPES, [0, 1, 2, 3, 4, 5, 6, 7, 8, 11, 12])}
ALL_CODES = [0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12]  # every dtype but Complex64 (9)
STORAGE = {0: np.float32, 1: np.float16, 2: np.uint8, 3: np.int32, 4: np.int16, 5: np.uint32, 6: np.uint16,
           7: np.bool_, 8: np.int8, 10: np.uint16, 11: np.int64, 12: np.uint64}  # BFloat16 bits in uint16
INT_RANGE = {2: (0, 255), 3: (-2**31, 2**31 - 1), 4: (-2**15, 2**15 - 1), 5: (0, 2**32 - 1), 6: (0, 2**16 - 1),
             8: (-128, 127), 11: (-2**63, 2**63 - 1), 12: (0, 2**64 - 1)}


def bf16_bits(x32):
    u = x32.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(x32)] = 0x7FC0
    return r


def values(rng, code, n, dst_code=None, special=False):
    """Random values of dtype `code`; when converting float-likes to an integer dtype, kept inside the
    destination's range (outside it C++ leaves the conversion undefined)."""
    if code == 7:
        return rng.integers(0, 2, n).astype(np.bool_)
    if code in (0, 1, 10):
        v = (rng.standard_normal(n) * 40).astype(np.float32)
        whole = rng.random(n) < 0.1
        v[whole] = np.round(v[whole])
        if dst_code in INT_RANGE:
            # inside the destination's range after rounding to the source type too
            lo, hi = INT_RANGE[dst_code]
            v = np.clip(v, max(lo * 0.99, -60000), min(hi * 0.99, 60000)).astype(np.float32)
            if lo == 0:
                v = np.abs(v)
        elif special:
            pick = rng.integers(0, 16, n)
            v[pick == 0], v[pick == 1], v[pick == 2], v[pick == 3] = np.nan, np.inf, -np.inf, -0.0
        if code == 0:
            return v
        if code == 1:
            return v.astype(np.float16)
        return bf16_bits(v)
    lo, hi = INT_RANGE[code]
    dt = STORAGE[code]
    v = rng.integers(lo, hi, n, dtype=dt, endpoint=True)
    if n:  # values at and around the float rounding boundaries
        v[:: max(1, n // 7)] = np.array(16842753 if np.iinfo(dt).max >= 16842753 else np.iinfo(dt).max, dtype=dt)
    return v


def same(a, b):
    return a.shape == b.shape and (a.tobytes() == b.tobytes() or np.array_equal(a, b, equal_nan=True))


@pytest.mark.parametrize("src", ALL_CODES)
def test_astype_matches_reference(port, ref, src):
    rng = np.random.default_rng(100 + src)
    for dst in ALL_CODES:
        for trial in range(4):
            shape = [int(v) for v in rng.integers(1, 7, int(rng.integers(1, 4)))]
            base = values(rng, src, int(np.prod(shape)) * 2, dst_code=dst, special=(dst not in INT_RANGE))
            x = base[: int(np.prod(shape))].reshape(shape)
            views = [x, x.T, x[..., ::2]] if x.ndim > 1 else [x, base[::2][: x.size]]
            for v in views:
                for mc in (True, False):
                    a = port.astype(v, STORAGE[dst], make_contig=mc, src_code=src, dst_code=dst)
                    b = ref.astype(v, STORAGE[dst], make_contig=mc, src_code=src, dst_code=dst)
                    assert same(np.ascontiguousarray(a), np.ascontiguousarray(b)), (src, dst, v.shape, v.strides, mc)
        # broadcast (stride-0) source axis kept by make_contig=False
        xb = np.broadcast_to(values(rng, src, 5, dst_code=dst), (3, 5))
        a = port.astype(xb, STORAGE[dst], make_contig=False, src_code=src, dst_code=dst)
        b = ref.astype(xb, STORAGE[dst], make_contig=False, src_code=src, dst_code=dst)
        assert same(np.ascontiguousarray(a), np.ascontiguousarray(b)), (src, dst, "broadcast")


def test_exp_and_sqrt_match_reference(port, ref):
    rng = np.random.default_rng(7)
    for op in ("exp", "sqrt"):
        for dt in (np.float32, np.float16):
            for trial in range(30):
                shape = [int(v) for v in rng.integers(1, 9, int(rng.integers(1, 4)))]
                x = (rng.standard_normal(int(np.prod(shape)) * 2) * 4).astype(dt)
                if op == "sqrt":
                    x = np.abs(x)
                x[::11] = np.array(np.nan, dtype=dt)
                v = x[: int(np.prod(shape))].reshape(shape)
                for view in (v, v.T):
                    assert same(port.unary(op, view), ref.unary(op, view)), (op, dt, shape)


@pytest.mark.parametrize("code", ALL_CODES)
def test_equal_matches_reference(port, ref, code):
    rng = np.random.default_rng(11 + code)
    for trial in range(30):
        dims = int(rng.integers(1, 5))
        out = [int(v) for v in rng.integers(1, 6, dims)]
        sa = [v if rng.random() < 0.6 else 1 for v in out][int(rng.integers(0, dims)):] or [1]
        sb = [v if rng.random() < 0.6 else 1 for v in out]
        a = values(rng, code, int(np.prod(sa)), special=True).reshape(sa)
        b = values(rng, code, int(np.prod(sb)), special=True).reshape(sb)
        b.reshape(-1)[: min(a.size, b.size) // 2] = a.reshape(-1)[: min(a.size, b.size) // 2]  # some equal pairs
        x = port.binary("equal", a, b, dtype_code=code)
        y = ref.binary("equal", a, b, dtype_code=code)
        assert same(x, y), (code, sa, sb)


def _collapse_case(rng):
    dims = int(rng.integers(0, 9))
    shape = [int(v) for v in rng.choice([1, 1, 2, 3, 5, 7, 64, 65536, 40000], dims)]
    n = int(rng.integers(1, 4))
    rows = []
    for _ in range(n):
        kind = rng.integers(0, 3)
        st, acc = [0] * dims, 1
        for i in range(dims - 1, -1, -1):
            if kind == 0:
                st[i] = acc & 0xFFFFFFFF
            elif kind == 1:
                st[i] = 0 if rng.random() < 0.4 else acc & 0xFFFFFFFF
            else:
                st[i] = int(rng.integers(0, 100))
            acc *= shape[i] + (1 if kind == 2 and rng.random() < 0.3 else 0)
        rows.append([0 if shape[i] == 1 else st[i] for i in range(dims)])
    return shape, rows


def test_pointwise_collapse_matches_reference(port, ref):
    rng = np.random.default_rng(12)
    for trial in range(3000):
        shape, rows = _collapse_case(rng)
        try:
            want = ref.pointwise_collapse(shape, rows)
        except ValueError:
            with pytest.raises(ValueError):
                port.pointwise_collapse(shape, rows)
            continue
        assert port.pointwise_collapse(shape, rows) == want, (shape, rows)


def test_product_pointwise_collapse_matches_oracle(port):
    from matrix_b200 import _abi

    L = _abi.lib()
    rng = np.random.default_rng(13)
    for trial in range(3000):
        shape, rows = _collapse_case(rng)
        n, d = len(rows), len(shape)
        flat = (C.c_uint32 * max(1, n * d))(*[v for r in rows for v in r])
        cs = _abi.u32_array([])
        cst = _abi.u32_array([], 3 * _abi.MAX_DIMS)
        k = L.mtxc_pointwise_collapse(_abi.u32_array(shape, max(d, 1)), d, flat, n, cs, cst)
        try:
            want = port.pointwise_collapse(shape, rows)
        except ValueError:
            assert k == 0xFFFFFFFF
            continue
        got = (k, list(cs[:k]), [list(cst[i * 8:i * 8 + k]) for i in range(n)])
        assert got == want, (shape, rows)
    assert L.mtxc_pointwise_collapse(_abi.u32_array([2] * 8, 9), 9, None, 0, _abi.u32_array([]), None) == 0xFFFFFFFF


@pytest.mark.parametrize("code", ALL_CODES)
def test_pointwise_backends_match_reference(port, ref, code):
    rng = np.random.default_rng(14 + code)
    for trial in range(25):
        dims = int(rng.integers(1, 5))
        out = [int(v) for v in rng.integers(1, 6, dims)]
        shapes = [[v if rng.random() < 0.7 else 1 for v in out][int(rng.integers(0, dims)):] or [1] for _ in range(3)]
        mk = [values(rng, code, int(np.prod(s)), special=True).reshape(s) for s in shapes]
        cond = rng.integers(0, 2, int(np.prod(shapes[0]))).astype(np.bool_).reshape(shapes[0])
        mk[1] = mk[1] if mk[1].ndim < 2 else mk[1].T.copy().T  # a strided copy keeps the same values
        cases = [("greater", mk[:2]), ("less", mk[:2]), ("where", [cond, mk[1], mk[2]]), ("floor", [mk[0]]),
                 ("full", [mk[2]])]
        if code == 7:
            cases.append(("logical_and", mk[:2]))
        for op, ins in cases:
            x = port.pointwise(op, ins, dtype_code=code)
            y = ref.pointwise(op, ins, dtype_code=code)
            assert same(x, y), (op, code, [i.shape for i in ins])


@pytest.mark.parametrize("code", ALL_CODES)
def test_stat_compositions_match_reference(port, ref, code):
    """mean / rms / norm composed from the primitives (mul, sum, astype, scalar division, sqrt) give
    the same bits through the restatement and through the reference's own loops."""
    rng = np.random.default_rng(60 + code)
    for shape, axis in (([4, 300], 1), ([300, 3], 0), ([2, 3, 50], 1), ([5], 0), ([3, 0], 1)):
        x = values(rng, code, int(np.prod(shape)), special=False).reshape(shape)
        for kind in ("mean", "rms", "norm"):
            for keep in (False, True):
                a, ca = port.stat(kind, x, axis, keep, dtype_code=code)
                b, cb = ref.stat(kind, x, axis, keep, dtype_code=code)
                assert ca == cb and same(a, b), (code, kind, shape, axis, keep)


def test_stat_output_dtypes(port):
    """The product's mtxc_reduce_stat_dtype equals the dtype the composition ends in."""
    from matrix_b200 import _abi

    L = _abi.lib()
    rng = np.random.default_rng(61)
    for code in ALL_CODES:
        for n in (5, 65504, 65505):
            x = values(rng, code, n).reshape(1, n)
            for k, kind in enumerate(("mean", "rms", "norm")):
                _, oc = port.stat(kind, x, 1, dtype_code=code)
                assert L.mtxc_reduce_stat_dtype(k, code, n) == oc, (code, n, kind)
    assert L.mtxc_reduce_stat_dtype(0, 9, 4) == -1 and L.mtxc_reduce_stat_dtype(3, 0, 4) == -1


def test_arctan2_and_arcsin_match_reference(port, ref):
    """arctan2 / arcsin (inputs cast to Float by the frontend): the restatement's loops equal the
    reference's own backends (std::atan2 / std::asin in float), incl. zeros, infinities, NaN and |x| > 1."""
    rng = np.random.default_rng(21)
    a = (rng.standard_normal((33, 65)) * 3).astype(np.float32)
    b = (rng.standard_normal((65,)) * 3).astype(np.float32)
    a[0, :8] = [0.0, -0.0, 0.0, -0.0, np.inf, -np.inf, np.nan, 1.0]
    b[:8] = [0.0, 0.0, -0.0, -0.0, np.inf, np.inf, 1.0, np.nan]
    for x, y in ((a, b), (a[:, ::2], b[::2]), (a.T.copy()[:5], a.T.copy()[5:10])):
        got, want = port.pointwise("arctan2", [x, y]), ref.pointwise("arctan2", [x, y])
        assert got.dtype == np.float32 and got.tobytes() == want.tobytes()
    x = rng.uniform(-1.2, 1.2, (7, 300)).astype(np.float32)
    x[0, :6] = [1.0, -1.0, 0.0, -0.0, np.nan, np.inf]
    for v in (x, x[:, 1::3], x[3]):
        assert port.pointwise("arcsin", [v]).tobytes() == ref.pointwise("arcsin", [v]).tobytes()


@pytest.mark.parametrize("code", [0, 1, 2, 3, 4, 5, 6, 8, 10, 11, 12])
def test_arange_matches_reference(port, ref, code):
    """arange's generator (integers through uint64 arithmetic, float-likes as float(start) + float(i) *
    float(step) without contraction) equals the reference's arange_backend_cpu for every dtype but Bool,
    which the reference's frontend refuses (Matrix.mm:13597) and the restatement with it."""
    dt = STORAGE[code]
    cases = [(0, 1, 0), (0, 1, 1), (3, 2, 1000), (-7, 3, 4099), (100, -1, 300), (0.5, 0.25, 70000),
             (-1e3, 0.1, 20001), (1, 7, 1 << 20)]
    for start, step, n in cases:
        if code in (0, 1, 10):
            s32, t32 = np.float32(start), np.float32(step)
            if code == 0:
                s, t = s32, t32
            elif code == 1:
                s, t = np.float16(start), np.float16(step)
            else:
                s, t = bf16_bits(np.array([s32]))[0], bf16_bits(np.array([t32]))[0]
        else:
            s = np.array(int(start)).astype(np.int64).astype(dt)
            t = np.array(int(step)).astype(np.int64).astype(dt)
        got = port.arange(s, t, n, dt, dtype_code=code)
        want = ref.arange(s, t, n, dt, dtype_code=code)
        assert got.tobytes() == want.tobytes(), (code, start, step, n)
    with pytest.raises(ValueError):
        port.arange(True, True, 4, np.bool_)
