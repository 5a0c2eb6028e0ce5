"""Python access to the CPU oracle (test infrastructure only).

Two interchangeable evaluators with the same interface:

* ``port()``      oracle/liboracle.so, the restatement in oracle/oracle.cpp;
* ``reference()`` oracle/_ref/libmtx_ref.so, the reference's own CPU loops and shape helpers
                  compiled by oracle/build_ref.py (None when it was not built).

The frontends here mirror the reference's graph-building methods (output shape, contiguous
output strides, collapse metadata) so a test states an op the way the reference's user would:
``ev.reduce("sum", x, axis=-1)`` is ``x.sum(-1)`` evaluated with ``eval_cpu()``.
Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libmtx_ref.so"

MAX_DIMS = 8
UINT32_MAX = 0xFFFFFFFF
INT32_MAX = 0x7FFFFFFF

# dtype codes, matrix.h:35-51
DTYPES = {
    np.dtype(np.float32): 0, np.dtype(np.uint8): 2, np.dtype(np.int32): 3, np.dtype(np.int16): 4,
    np.dtype(np.uint32): 5, np.dtype(np.uint16): 6, np.dtype(np.int8): 8, np.dtype(np.int64): 11,
    np.dtype(np.uint64): 12, np.dtype(np.float16): 1, np.dtype(np.bool_): 7,
}
BF16 = 10  # numpy has no bfloat16: its bits travel as uint16 with an explicit dtype code
# numpy storage of each dtype code (BFloat16 bits in uint16)
STORAGE = {0: np.float32, 1: np.float16, 2: np.uint8, 3: np.int32, 4: np.int16, 5: np.uint32, 6: np.uint16,
           7: np.bool_, 8: np.int8, 10: np.uint16, 11: np.int64, 12: np.uint64}
REDUCE_OPS = {"sum": 0, "max": 1, "min": 2, "argmax": 3, "argmin": 4}
BINARY_OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "max": 4, "min": 5, "equal": 6}
UNARY_OPS = {"exp": 0, "sqrt": 1}
POINTWISE_OPS = {"greater": 0, "less": 1, "logical_and": 2, "where": 3, "floor": 4, "full": 5, "arctan2": 6,
                 "arcsin": 7}

U32P = C.POINTER(C.c_uint32)


def _arr(vals, n=MAX_DIMS):
    a = (C.c_uint32 * n)()
    for i, v in enumerate(vals):
        a[i] = int(v) & 0xFFFFFFFF
    return a


def row_major(shape):
    strides, acc = [0] * len(shape), 1
    for i in range(len(shape) - 1, -1, -1):
        strides[i] = acc & 0xFFFFFFFF  # size_m arithmetic
        acc *= int(shape[i])
    return strides


def elem_strides(x: np.ndarray):
    return [s // x.itemsize for s in x.strides]


class CpuEval:
    """ctypes wrapper over one of the two oracle libraries."""

    def __init__(self, path: Path, prefix: str, threaded: bool):
        self.path = path
        self.prefix = prefix
        self.threaded = threaded
        self.lib = C.CDLL(str(path))
        self.threads = int(os.environ.get("ORACLE_THREADS", "1"))
        L = self.lib
        u32, u64, i32 = C.c_uint32, C.c_uint64, C.c_int
        vp = C.c_void_p
        self._f = {}

        def fn(name, res, args):
            f = getattr(L, prefix + name)
            f.restype, f.argtypes = res, args
            self._f[name] = f

        fn("collapse1", u32, [U32P, U32P, u32, u64, U32P, U32P])
        fn("collapse2", u32, [U32P, U32P, U32P, u32, u64, U32P, U32P, U32P])
        fn("collapse3", u32, [U32P, U32P, U32P, U32P, u32, u64, U32P, U32P, U32P, U32P])
        fn("collapse_reduce1", u32, [U32P, U32P, u32, i32, i32, u64, U32P, U32P])
        fn("collapse_reduce2", u32, [U32P, U32P, U32P, u32, i32, i32, i32, u64, U32P, U32P, U32P])
        fn("collapse_reduce3", u32, [U32P, U32P, U32P, U32P, u32, i32, i32, u64, U32P, U32P, U32P, U32P])
        fn("broadcast_shapes", i32, [U32P, U32P, i32, U32P, U32P, i32, U32P, U32P, U32P, U32P, U32P, U32P])
        fn("promote", i32, [i32, i32])
        extra = [i32] if threaded else []
        fn("reduce", i32, [i32, i32, vp, vp, u32, u32, u32, U32P, U32P, U32P, u64] + extra)
        fn("broadcast", i32, [i32, i32, vp, vp, vp, u32, U32P, U32P, U32P, u64] + extra)
        fn("exp", i32, [i32, vp, vp, u32, U32P, U32P, U32P, u64] + extra)
        fn("unary", i32, [i32, i32, vp, vp, u32, U32P, U32P, U32P, u64] + extra)
        fn("astype", i32, [i32, i32, vp, vp, u32, U32P, U32P, U32P, u64] + extra)
        fn("pointwise_collapse", u32, [U32P, u32, U32P, u32, U32P, U32P])
        fn("pointwise", i32, [i32, i32, vp, C.POINTER(vp), u32, u32, U32P, U32P, u64] + extra)
        fn("arange", i32, [i32, vp, vp, vp, u64])
        if prefix == "orc_":
            fn("sum_flat", i32, [i32, vp, vp, u64])
        if prefix == "ref_":
            fn("equal", i32, [i32, vp, vp, vp, u32, U32P, U32P, U32P, U32P, u64])

    # -- shape folding ---------------------------------------------------------------------
    def collapse(self, shape, *strides, cap=INT32_MAX):
        n = len(strides)
        o = [_arr([]) for _ in range(n + 1)]
        args = [_arr(shape)] + [_arr(s) for s in strides] + [len(shape), cap] + o
        k = self._f[f"collapse{n}"](*args)
        return k, [list(a[:k]) for a in o]

    def collapse_reduce(self, shape, *strides, axis, keep=False, outer=None, cap=UINT32_MAX):
        n = len(strides)
        o = [_arr([]) for _ in range(n + 1)]
        args = [_arr(shape)] + [_arr(s) for s in strides] + [len(shape), axis, int(keep)]
        if n == 2:
            args.append(int(bool(outer)))
        args += [cap] + o
        k = self._f[f"collapse_reduce{n}"](*args)
        return k, [list(a[:k]) for a in o]

    def broadcast_shapes(self, shape1, strides1, shape2, strides2):
        od = max(len(shape1), len(shape2))
        outs = [_arr([]) for _ in range(6)]
        rc = self._f["broadcast_shapes"](_arr(shape1), _arr(strides1), len(shape1), _arr(shape2), _arr(strides2),
                                         len(shape2), *outs)
        if rc != 0:
            raise ValueError("Incompatible shapes for broadcasting")
        return [list(a[:od]) for a in outs]  # out_shape, out_strides, a_shape, a_strides, b_shape, b_strides

    def promote(self, a, b):
        return self._f["promote"](a, b)

    # -- frontends (the reference's graph-building metadata) -------------------------------
    def reduce_meta(self, shape, strides, axis, keepdims=False):
        """matrix::sum/max/... (Matrix.mm:15071-15097): output shape, row-major output strides,
        collapse_dims_reduce(shape, out.strides, in.strides, dims, axis, false, !keepdims, UINT32_MAX)."""
        dims = len(shape)
        if axis < 0:
            axis += dims
        if keepdims:
            out_shape = list(shape)
            out_shape[axis] = 1
        else:
            out_shape = list(shape[:axis]) + list(shape[axis + 1:])
        out_strides = row_major(out_shape)
        so = out_strides + [0] * (dims - len(out_strides))
        k, (cshape, s_out, s_in) = self.collapse_reduce(shape, so, strides, axis=axis, keep=False,
                                                        outer=not keepdims, cap=UINT32_MAX)
        return dict(out_shape=out_shape, cdims=k, shape=cshape, s_out=s_out, s_in=s_in,
                    rstride=int(strides[axis]), rlen=int(shape[axis]))

    def binary_meta(self, shape_a, strides_a, shape_b, strides_b):
        """operator+ & co. (Matrix.mm:8312-8331): broadcast_shapes, then collapse_dims over
        (desc_a.shape, desc_a.strides, desc_b.strides, result.strides) with cap INT32_MAX."""
        out_shape, out_strides, a_shape, a_strides, b_shape, b_strides = self.broadcast_shapes(
            shape_a, strides_a, shape_b, strides_b)
        k, (cshape, sa, sb, sr) = self.collapse(a_shape, a_strides, b_strides, out_strides, cap=INT32_MAX)
        return dict(out_shape=out_shape, cdims=k, shape=cshape, sa=sa, sb=sb, sr=sr)

    def unary_meta(self, shape, strides):
        """matrix::exp (Matrix.mm:6934-6947): collapse_dims(shape, out.strides, in.strides)."""
        k, (cshape, so, si) = self.collapse(shape, row_major(shape), strides, cap=INT32_MAX)
        return dict(out_shape=list(shape), cdims=k, shape=cshape, s_out=so, s_in=si)

    # -- evaluation --------------------------------------------------------------------------
    def _thr(self):
        return [self.threads] if self.threaded else []

    def reduce_raw(self, op, x_base: np.ndarray, offset: int, meta, dtype_code=None):
        total = int(np.prod(meta["out_shape"], dtype=np.int64)) if meta["out_shape"] else 1
        opc = REDUCE_OPS[op]
        odt = np.int32 if opc >= 3 else x_base.dtype
        out = np.empty(max(total, 1), dtype=odt)
        ptr = x_base.ctypes.data + offset * x_base.itemsize
        code = DTYPES[x_base.dtype] if dtype_code is None else dtype_code
        rc = self._f["reduce"](opc, code, out.ctypes.data, ptr, meta["rstride"] & 0xFFFFFFFF,
                               meta["rlen"], meta["cdims"], _arr(meta["shape"]), _arr(meta["s_out"]),
                               _arr(meta["s_in"]), total, *self._thr())
        if rc != 0:
            raise RuntimeError(f"{self.prefix}reduce failed")
        return out[:total].reshape(meta["out_shape"])

    def sum_flat(self, x: np.ndarray, dtype_code=None):
        """x.sum() for a contiguous x of any size: one sequential sum over every element in memory order
        (the restatement only; the reference's own loop cannot count past 2^32 - 1 elements)."""
        if "sum_flat" not in self._f:
            raise NotImplementedError("sum_flat is the restatement's (port()) only")
        if not x.flags.c_contiguous:
            raise ValueError("sum_flat needs a contiguous array")
        out = np.zeros(1, dtype=x.dtype)
        code = DTYPES[x.dtype] if dtype_code is None else dtype_code
        if self._f["sum_flat"](code, out.ctypes.data, x.ctypes.data, x.size) != 0:
            raise RuntimeError("orc_sum_flat failed")
        return out[0]

    def reduce(self, op, x: np.ndarray, axis: int, keepdims=False, dtype_code=None):
        """x.op(axis, keepdims).eval_cpu() for a (possibly strided) numpy view x.  dtype_code
        overrides the code numpy's dtype implies (BF16 data held as uint16)."""
        base, offset = _base_and_offset(x)
        meta = self.reduce_meta(list(x.shape), elem_strides(x), axis, keepdims)
        return self.reduce_raw(op, base, offset, meta, dtype_code)

    def binary_raw(self, op, a_base, a_off, b_base, b_off, meta, dtype_code=None):
        total = int(np.prod(meta["out_shape"], dtype=np.int64)) if meta["out_shape"] else 1
        out = np.empty(max(total, 1), dtype=a_base.dtype)
        code = DTYPES[a_base.dtype] if dtype_code is None else dtype_code
        pa = a_base.ctypes.data + a_off * a_base.itemsize
        pb = b_base.ctypes.data + b_off * b_base.itemsize
        if op == "equal" and self.prefix == "ref_":
            # the reference's own equal loop (matrix::equal_backend), same collapse_dims_3 metadata
            rc = self._f["equal"](code, out.ctypes.data, pa, pb, meta["cdims"], _arr(meta["shape"]),
                                  _arr(meta["sa"]), _arr(meta["sb"]), _arr(meta["sr"]), total)
        else:
            rc = self._f["broadcast"](BINARY_OPS[op], code, out.ctypes.data, pa, pb, meta["cdims"], _arr(meta["sr"]),
                                      _arr(meta["sa"]), _arr(meta["sb"]), total, *self._thr())
        if rc != 0:
            raise RuntimeError(f"{self.prefix}broadcast failed")
        return out[:total].reshape(meta["out_shape"])

    def binary(self, op, a: np.ndarray, b: np.ndarray, dtype_code=None):
        """(a op b).eval_cpu() with both operands already of the same dtype."""
        assert a.dtype == b.dtype
        ab, ao = _base_and_offset(a)
        bb, bo = _base_and_offset(b)
        meta = self.binary_meta(list(a.shape), elem_strides(a), list(b.shape), elem_strides(b))
        return self.binary_raw(op, ab, ao, bb, bo, meta, dtype_code)

    def exp(self, x: np.ndarray):
        base, offset = _base_and_offset(x)
        meta = self.unary_meta(list(x.shape), elem_strides(x))
        total = int(np.prod(x.shape, dtype=np.int64)) if x.shape else 1
        out = np.empty(max(total, 1), dtype=np.float32)
        rc = self._f["exp"](0, out.ctypes.data, base.ctypes.data + offset * base.itemsize, meta["cdims"],
                            _arr(meta["shape"]), _arr(meta["s_out"]), _arr(meta["s_in"]), total, *self._thr())
        if rc != 0:
            raise RuntimeError(f"{self.prefix}exp failed")
        return out[:total].reshape(x.shape)


    def unary(self, op, x: np.ndarray, dtype_code=None):
        """matrix::exp / matrix::sqrt on a Float or Float16 view (the frontends promote other
        dtypes with astype first)."""
        base, offset = _base_and_offset(x)
        meta = self.unary_meta(list(x.shape), elem_strides(x))
        total = int(np.prod(x.shape, dtype=np.int64)) if x.shape else 1
        out = np.empty(max(total, 1), dtype=x.dtype)
        code = DTYPES[x.dtype] if dtype_code is None else dtype_code
        rc = self._f["unary"](UNARY_OPS[op], code, out.ctypes.data, base.ctypes.data + offset * base.itemsize,
                              meta["cdims"], _arr(meta["shape"]), _arr(meta["s_out"]), _arr(meta["s_in"]), total,
                              *self._thr())
        if rc != 0:
            raise RuntimeError(f"{self.prefix}unary failed")
        return out[:total].reshape(x.shape)

    def astype(self, x: np.ndarray, dst, make_contig=True, src_code=None, dst_code=None):
        """x.astype(dst, make_contig).eval_cpu() (Matrix.mm:8384-8398, 8400-8412).  With make_contig
        the output is row-major; otherwise it takes the input's strides (broadcast axes included),
        as the promotion path's astype(common) does.  dst: a numpy dtype (the output's storage);
        src_code / dst_code override the dtype codes (BFloat16 bits held as uint16)."""
        base, offset = _base_and_offset(x)
        shape, s_in = list(x.shape), elem_strides(x)
        s_out = row_major(shape) if make_contig else list(s_in)
        total = int(np.prod(shape, dtype=np.int64)) if shape else 1
        span = 1 + sum((e - 1) * st for e, st in zip(shape, s_out)) if total else 0
        out = np.zeros(max(span, 1), dtype=dst)
        sc = DTYPES[x.dtype] if src_code is None else src_code
        dc = DTYPES[np.dtype(dst)] if dst_code is None else dst_code
        src_ptr = base.ctypes.data + offset * base.itemsize
        if self.prefix == "ref_":  # copyCPUinplaceTypeCasted collapses the metadata itself
            rc = self._f["astype"](dc, sc, out.ctypes.data, src_ptr, len(shape), _arr(shape), _arr(s_out),
                                   _arr(s_in), total)
        else:
            k, (cshape, so, si) = self.collapse(shape, s_out, s_in, cap=INT32_MAX)
            rc = self._f["astype"](dc, sc, out.ctypes.data, src_ptr, k, _arr(cshape), _arr(so), _arr(si), total,
                                   *self._thr())
        if rc != 0:
            raise RuntimeError(f"{self.prefix}astype failed")
        if total == 0:
            return np.zeros(shape, dtype=dst)
        return np.lib.stride_tricks.as_strided(out, shape=shape, strides=[st * out.itemsize for st in s_out])

    def pointwise_collapse(self, out_shape, in_strides):
        """make_pointwise's collapse (Matrix.mm:13537-13555); in_strides: one list per input,
        right-aligned to the output rank, 0 on broadcast axes."""
        n, d = len(in_strides), len(out_shape)
        flat = (C.c_uint32 * max(1, n * d))(*[int(v) & 0xFFFFFFFF for row in in_strides for v in row])
        cshape = _arr([])
        cstr = (C.c_uint32 * (3 * MAX_DIMS))()
        k = self._f["pointwise_collapse"](_arr(out_shape, max(d, 1)), d, flat, n, cshape, cstr)
        if k == UINT32_MAX:
            raise ValueError("pointwise collapse refused the shape")
        return k, list(cshape[:k]), [list(cstr[i * MAX_DIMS:i * MAX_DIMS + k]) for i in range(n)]

    def pointwise_meta(self, inputs):
        """pointwise_shape + make_pointwise (Matrix.mm:13497-13556) for numpy views: the broadcast
        output shape, each input's right-aligned strides (0 where its extent is 1) and the collapse."""
        rank = max((x.ndim for x in inputs), default=0)
        shape = [1] * rank
        for x in inputs:
            for d, m in enumerate(x.shape):
                n = shape[rank - x.ndim + d]
                if n == 1:
                    shape[rank - x.ndim + d] = m
                elif m != 1 and n != m:
                    raise ValueError("incompatible pointwise broadcast shapes")
        rows = []
        for x in inputs:
            st = [0] * rank
            for d, (m, s) in enumerate(zip(x.shape, elem_strides(x))):
                st[rank - x.ndim + d] = 0 if m == 1 else s
            rows.append(st)
        k, cshape, cstr = self.pointwise_collapse(shape, rows)
        return dict(out_shape=shape, cdims=k, shape=cshape, strides=cstr)

    def pointwise(self, op, inputs, dtype_code=None):
        """greater / less / logical_and / where / floor / full / arctan2 / arcsin over numpy views already
        cast to their common dtype (cond of where: bool; Float for arctan2 / arcsin).  Returns the
        contiguous output."""
        meta = self.pointwise_meta(inputs)
        total = int(np.prod(meta["out_shape"], dtype=np.int64)) if meta["out_shape"] else 1
        data = inputs[-1]
        odt = (np.bool_ if op in ("greater", "less", "logical_and") else
               np.float32 if op in ("arctan2", "arcsin") else data.dtype)
        out = np.zeros(max(total, 1), dtype=odt)
        code = DTYPES[data.dtype] if dtype_code is None else dtype_code
        if op == "logical_and":
            code = DTYPES[np.dtype(np.bool_)]
        ptrs = []
        for x in inputs:
            b, o = _base_and_offset(x)
            ptrs.append(b.ctypes.data + o * b.itemsize)
        arr = (C.c_void_p * 3)(*ptrs)
        st = (C.c_uint32 * (3 * MAX_DIMS))()
        for i, row in enumerate(meta["strides"]):
            for j, v in enumerate(row):
                st[i * MAX_DIMS + j] = v
        if total:
            rc = self._f["pointwise"](POINTWISE_OPS[op], code, out.ctypes.data, arr, len(inputs), meta["cdims"],
                                      _arr(meta["shape"]), st, total, *self._thr())
            if rc != 0:
                raise RuntimeError(f"{self.prefix}pointwise failed")
        return out[:total].reshape(meta["out_shape"])


    def arange(self, start, step, count: int, dtype, dtype_code=None):
        """arange's CPU backend: count elements start + i * step of `dtype` (start and step already
        converted to it, as matrix::scalar does)."""
        dt = np.dtype(dtype)
        a = np.array([start], dtype=dt)
        b = np.array([step], dtype=dt)
        out = np.zeros(max(count, 1), dtype=dt)
        code = DTYPES.get(dt, -1) if dtype_code is None else dtype_code
        if self._f["arange"](code, out.ctypes.data, a.ctypes.data, b.ctypes.data, count) != 0:
            raise ValueError(f"{self.prefix}arange refused dtype {dt}")
        return out[:count]

    # -- mean / rms / norm: the reference's compositions (Matrix.mm:15220-15276) ------------
    def _scalar_type(self, value: float, code: int) -> int:
        """scalar_operand_type(float scalar, code) (matrix.h:1815-1822) for a float scalar."""
        if code in (0, BF16, 9):
            return code
        if code == 1:
            return 1 if -65504 <= value <= 65504 else 0
        return 0

    def _sqrt(self, v: np.ndarray, code: int):
        """matrix::sqrt(v): astype to promote_types(code, Float16), then the sqrt loop."""
        oc = self.promote(code, 1)
        if oc != code:
            v = self.astype(v, STORAGE[oc], src_code=code, dst_code=oc)
        return self.unary("sqrt", np.asarray(v), dtype_code=oc), oc

    def _div_by(self, s: np.ndarray, code: int, value: float):
        """s / value with the reference's scalar rules (operator/(matrix, T), matrix.h:1868)."""
        sc = self._scalar_type(value, code)
        common = self.promote(code, sc)
        lhs = s if code == common else self.astype(s, STORAGE[common], src_code=code, dst_code=common)
        rhs = self.astype(np.array(value, dtype=np.float32), STORAGE[sc], dst_code=sc)  # matrix::scalar
        if sc != common:
            rhs = self.astype(rhs, STORAGE[common], src_code=sc, dst_code=common)
        return self.binary("div", np.asarray(lhs), np.asarray(rhs), dtype_code=common), common

    def stat(self, kind: str, x: np.ndarray, axis: int, keepdims=False, dtype_code=None):
        """x.mean / rms / norm(axis, keepdims).eval_cpu() as the reference composes them from its
        primitives.  Returns (result, result dtype code)."""
        code = DTYPES[x.dtype] if dtype_code is None else dtype_code
        data = self.binary("mul", x, x, dtype_code=code) if kind in ("rms", "norm") else x
        s = self.reduce("sum", data, axis, keepdims, dtype_code=code)
        if kind == "norm":
            return self._sqrt(s, code)
        n = x.shape[axis]
        m, mcode = self._div_by(s, code, float(np.float32(n)))
        if kind == "mean":
            return m, mcode
        return self._sqrt(m, mcode)


def _base_and_offset(x: np.ndarray):
    """The flat base buffer of a view and the view's element offset into it."""
    base = x
    while isinstance(base.base, np.ndarray):
        base = base.base
    if not (base.flags.c_contiguous or base.flags.f_contiguous):
        base = np.ascontiguousarray(base)
    flat = base.reshape(-1, order="A") if base.ndim != 1 else base
    off_bytes = x.__array_interface__["data"][0] - flat.__array_interface__["data"][0]
    assert off_bytes % x.itemsize == 0
    if flat.dtype != x.dtype:
        flat = flat.view(x.dtype)
    return flat, off_bytes // x.itemsize


_PORT = None
_REF = None


def port() -> CpuEval:
    global _PORT
    if _PORT is None:
        if not PORT_LIB.exists():
            raise FileNotFoundError(f"{PORT_LIB} is missing: run `python oracle/build.py`")
        _PORT = CpuEval(PORT_LIB, "orc_", threaded=True)
    return _PORT


def reference() -> CpuEval | None:
    global _REF
    if _REF is None:
        if not REF_LIB.exists():
            return None
        _REF = CpuEval(REF_LIB, "ref_", threaded=False)
    return _REF
