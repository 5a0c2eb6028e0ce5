"""Python driver of the C ABI on device tensors.

The functions here mirror the reference's frontends for the hot path: they compute the same
metadata the reference's graph-building methods cache on their primitive, using the library's
own shape folding (mtxc_collapse_dims*, mtxc_broadcast_shapes), and then call the backend entry
point with it.  ``reduce("sum", x, -1)`` is the reference's ``x.sum(-1)`` followed by
``eval()`` on the GPU (Matrix.mm:15071-15186); ``binary("add", a, b)`` is ``a + b``
(Matrix.mm:8312-8331, 7709-7868).  PyTorch only provides device memory and streams.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _abi
from ._abi import check, lib, u32_array

UINT32_MAX = 0xFFFFFFFF
INT32_MAX = 0x7FFFFFFF

TORCH_DTYPES = {
    torch.float32: 0, torch.float16: 1, torch.uint8: 2, torch.int32: 3, torch.int16: 4, torch.uint32: 5,
    torch.uint16: 6, torch.bool: 7, torch.int8: 8, torch.bfloat16: 10, torch.int64: 11, torch.uint64: 12,
}


def dtype_code(t: torch.dtype) -> int:
    try:
        return TORCH_DTYPES[t]
    except KeyError:
        raise _abi.MtxcError(_abi.ERR_UNSUPPORTED_DTYPE, f"no kernel for {t}") from None


def init(device: int = 0, stream: torch.cuda.Stream | None = None) -> None:
    """Binds the calling thread to `device` and makes `stream` (default: torch's current
    stream on that device) the stream the backend launches on."""
    check(lib().mtxc_init(int(device)))
    if stream is None:
        stream = torch.cuda.current_stream(device)
    check(lib().mtxc_set_stream(stream.cuda_stream))


def set_stream(stream: torch.cuda.Stream) -> None:
    check(lib().mtxc_set_stream(stream.cuda_stream))


def sync() -> None:
    check(lib().mtxc_sync())


def row_major(shape):
    strides, acc = [0] * len(shape), 1
    for i in range(len(shape) - 1, -1, -1):
        strides[i] = acc & 0xFFFFFFFF
        acc *= int(shape[i])
    return strides


# ------------------------------------------------------------------------------------------
# Frontend metadata
# ------------------------------------------------------------------------------------------
@dataclass
class ReduceMeta:
    out_shape: list
    cdims: int
    shape: list
    s_out: list
    s_in: list
    rstride: int
    rlen: int
    arrays: tuple = field(default=(), repr=False)


def reduce_meta(shape, strides, axis: int, keepdims: bool = False) -> ReduceMeta:
    """Output shape and collapse_dims_reduce(shape, out.strides, in.strides, dims, axis, false,
    !keepdims, UINT32_MAX), as matrix::sum / max / min / argmax / argmin build them
    (Matrix.mm:15071-15097, 14784-14810, 14927-14954, 16150-16180, 16305-16335)."""
    dims = len(shape)
    if dims == 0:
        raise ValueError("reduction of a 0-d tensor")
    if axis < 0:
        axis += dims
    if not 0 <= axis < dims:
        raise ValueError(f"axis {axis} out of range for rank {dims}")
    if keepdims:
        out_shape = list(shape)
        out_shape[axis] = 1
    else:
        out_shape = list(shape[:axis]) + list(shape[axis + 1:])
    out_strides = row_major(out_shape) + [0] * (dims - len(out_shape))
    o = [u32_array([]) for _ in range(3)]
    k = lib().mtxc_collapse_dims_reduce2(u32_array(shape), u32_array(out_strides), u32_array(strides), dims, axis, 0,
                                         int(not keepdims), UINT32_MAX, *o)
    arr = tuple(o)
    return ReduceMeta(out_shape, k, list(o[0][:k]), list(o[1][:k]), list(o[2][:k]), int(strides[axis]),
                      int(shape[axis]), arr)


@dataclass
class BinaryMeta:
    out_shape: list
    cdims: int
    shape: list
    sr: list
    sa: list
    sb: list
    arrays: tuple = field(default=(), repr=False)


def binary_meta(shape_a, strides_a, shape_b, strides_b) -> BinaryMeta:
    """broadcast_shapes, then collapse_dims(desc_a.shape, desc_a.strides, desc_b.strides,
    result.strides, dims, INT32_MAX), as operator+ - * / and matrix::max / min(a, b) do
    (Matrix.mm:8312-8382, 13363-13376, 14668-14682)."""
    od = max(len(shape_a), len(shape_b))
    outs = [u32_array([]) for _ in range(6)]
    rc = lib().mtxc_broadcast_shapes(u32_array(shape_a), u32_array(strides_a), len(shape_a), u32_array(shape_b),
                                     u32_array(strides_b), len(shape_b), *outs)
    if rc == _abi.ERR_SHAPE:
        raise ValueError("Incompatible shapes for broadcasting")
    check(rc)
    out_shape, out_strides, a_shape, a_strides, _b_shape, b_strides = outs
    o = [u32_array([]) for _ in range(4)]
    k = lib().mtxc_collapse_dims3(a_shape, a_strides, b_strides, out_strides, od, INT32_MAX, *o)
    return BinaryMeta(list(out_shape[:od]), k, list(o[0][:k]), list(o[3][:k]), list(o[1][:k]), list(o[2][:k]),
                      (o[0], o[3], o[1], o[2]))


@dataclass
class UnaryMeta:
    out_shape: list
    cdims: int
    shape: list
    s_out: list
    s_in: list
    arrays: tuple = field(default=(), repr=False)


def unary_meta(shape, strides) -> UnaryMeta:
    """collapse_dims(shape, out.strides, in.strides, dims, INT32_MAX) (Matrix.mm:6934-6947)."""
    o = [u32_array([]) for _ in range(3)]
    k = lib().mtxc_collapse_dims2(u32_array(shape), u32_array(row_major(shape)), u32_array(strides), len(shape),
                                  INT32_MAX, *o)
    return UnaryMeta(list(shape), k, list(o[0][:k]), list(o[1][:k]), list(o[2][:k]), tuple(o))


# ------------------------------------------------------------------------------------------
# Device ops
# ------------------------------------------------------------------------------------------
def _check_strides(x: torch.Tensor):
    st = x.stride()
    if any(s < 0 for s in st):
        raise ValueError("negative strides are not representable in the reference's size_m metadata")
    return list(st)


def reduce_launch(op: str, x_ptr: int, dtype: int, out_ptr: int, meta: ReduceMeta) -> None:
    shape, s_out, s_in = meta.arrays
    check(lib().mtxc_reduce(_abi.REDUCE_OPS[op], dtype, out_ptr, x_ptr, meta.rstride & 0xFFFFFFFF, meta.rlen,
                            meta.cdims, shape, s_out, s_in))


def reduce(op: str, x: torch.Tensor, axis: int, keepdims: bool = False, out: torch.Tensor | None = None,
           meta: ReduceMeta | None = None) -> torch.Tensor:
    """x.<op>(axis, keepdims) evaluated on the GPU through mtxc_reduce."""
    code = dtype_code(x.dtype)
    if meta is None:
        meta = reduce_meta(list(x.shape), _check_strides(x), axis, keepdims)
    odt = torch.int32 if op in ("argmax", "argmin") else x.dtype
    if out is None:
        out = torch.empty(meta.out_shape, dtype=odt, device=x.device)
    reduce_launch(op, x.data_ptr(), code, out.data_ptr(), meta)
    return out


CODE_TO_TORCH = {v: k for k, v in TORCH_DTYPES.items()}


def stat(kind: str, x: torch.Tensor, axis: int, keepdims: bool = False, meta: ReduceMeta | None = None):
    """x.mean / rms / norm(axis, keepdims) in one pass (mtxc_reduce_stat).  The output dtype is the
    one the reference's composition ends in (mtxc_reduce_stat_dtype)."""
    code = dtype_code(x.dtype)
    if meta is None:
        meta = reduce_meta(list(x.shape), _check_strides(x), axis, keepdims)
    oc = lib().mtxc_reduce_stat_dtype(_abi.STATS[kind], code, meta.rlen)
    out = torch.empty(meta.out_shape, dtype=CODE_TO_TORCH[oc], device=x.device)
    shape, s_out, s_in = meta.arrays
    check(lib().mtxc_reduce_stat(_abi.STATS[kind], code, out.data_ptr(), x.data_ptr(), meta.rstride & 0xFFFFFFFF,
                                 meta.rlen, meta.cdims, shape, s_out, s_in))
    return out


def binary_launch(op: str, a_ptr: int, b_ptr: int, dtype: int, out_ptr: int, meta: BinaryMeta) -> None:
    shape, sr, sa, sb = meta.arrays
    check(lib().mtxc_broadcast_binary(_abi.BINARY_OPS[op], dtype, out_ptr, a_ptr, b_ptr, meta.cdims, shape, sr, sa,
                                      sb))


MIXED_OPS = ("add", "sub", "mul", "div", "equal")


def binary(op: str, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
           meta: BinaryMeta | None = None) -> torch.Tensor:
    """a <op> b with broadcasting, evaluated through mtxc_broadcast_binary.  Operands of different
    dtypes are promoted as the reference does (promote_types, astype of both operands first), in one pass
    through mtxc_broadcast_binary_mixed: each operand is converted to the promoted dtype as it is read."""
    if a.dtype != b.dtype:
        if op not in MIXED_OPS:
            raise _abi.MtxcError(_abi.ERR_UNSUPPORTED_DTYPE, "max / min of mixed dtypes: cast one operand first")
        ca, cb = dtype_code(a.dtype), dtype_code(b.dtype)
        common = lib().mtxc_promote_types(ca, cb)
        if common in CODE_TO_TORCH:
            if meta is None:
                meta = binary_meta(list(a.shape), _check_strides(a), list(b.shape), _check_strides(b))
            if out is None:
                out = torch.empty(meta.out_shape, dtype=CODE_TO_TORCH[common], device=a.device)
            shape, sr, sa, sb = meta.arrays
            check(lib().mtxc_broadcast_binary_mixed(_abi.BINARY_OPS[op], common, ca, cb, out.data_ptr(),
                                                     a.data_ptr(), b.data_ptr(), meta.cdims, shape, sr, sa, sb))
            return out
        t = CODE_TO_TORCH[common]
        a = a if a.dtype == t else astype(a, t, make_contig=False)
        b = b if b.dtype == t else astype(b, t, make_contig=False)
        meta = None
    code = dtype_code(a.dtype)
    if meta is None:
        meta = binary_meta(list(a.shape), _check_strides(a), list(b.shape), _check_strides(b))
    if out is None:
        out = torch.empty(meta.out_shape, dtype=a.dtype, device=a.device)
    binary_launch(op, a.data_ptr(), b.data_ptr(), code, out.data_ptr(), meta)
    return out


def unary(op: str, x: torch.Tensor, out: torch.Tensor | None = None, meta: UnaryMeta | None = None) -> torch.Tensor:
    """matrix::exp(x) / matrix::sqrt(x) on a float32 or float16 tensor, through mtxc_unary."""
    code = dtype_code(x.dtype)
    if meta is None:
        meta = unary_meta(list(x.shape), _check_strides(x))
    if out is None:
        out = torch.empty(meta.out_shape, dtype=x.dtype, device=x.device)
    shape, so, si = meta.arrays
    check(lib().mtxc_unary(_abi.UNARY_OPS[op], code, out.data_ptr(), x.data_ptr(), meta.cdims, shape, so, si))
    return out


def exp(x: torch.Tensor, out: torch.Tensor | None = None, meta: UnaryMeta | None = None) -> torch.Tensor:
    """matrix::exp(x) evaluated through mtxc_unary."""
    return unary("exp", x, out, meta)


def astype(x: torch.Tensor, dtype: torch.dtype, make_contig: bool = True, out: torch.Tensor | None = None):
    """x.astype(dtype, make_contig) evaluated through mtxc_astype (Matrix.mm:8384-8412).  Without
    make_contig the output takes x's strides (broadcast axes included), as the promotion path does."""
    shape, s_in = list(x.shape), _check_strides(x)
    if out is None:
        out = (torch.empty(shape, dtype=dtype, device=x.device) if make_contig
               else torch.empty_strided(shape, s_in, dtype=dtype, device=x.device))
    s_out = _check_strides(out)
    o = [u32_array([]) for _ in range(3)]
    k = lib().mtxc_collapse_dims2(u32_array(shape), u32_array(s_out), u32_array(s_in), len(shape), INT32_MAX, *o)
    check(lib().mtxc_astype(dtype_code(dtype), dtype_code(x.dtype), out.data_ptr(), x.data_ptr(), k, *o))
    return out


@dataclass
class PointwiseMeta:
    out_shape: list
    cdims: int
    shape: list
    strides: list
    arrays: tuple = field(default=(), repr=False)


def pointwise_meta(shapes, strides) -> PointwiseMeta:
    """pointwise_shape + make_pointwise's collapse (Matrix.mm:13497-13556) for inputs given as
    (shape, strides) lists: the broadcast output shape, each input's right-aligned strides (0 where
    its extent is 1) collapsed by mtxc_pointwise_collapse."""
    rank = max((len(sh) for sh in shapes), default=0)
    out = [1] * rank
    for sh in shapes:
        for d, m in enumerate(sh):
            n = out[rank - len(sh) + d]
            if n == 1:
                out[rank - len(sh) + d] = m
            elif m != 1 and n != m:
                raise _abi.MtxcError(_abi.ERR_SHAPE, "incompatible pointwise broadcast shapes")
    rows = []
    for sh, st in zip(shapes, strides):
        r = [0] * rank
        for d, (m, s) in enumerate(zip(sh, st)):
            r[rank - len(sh) + d] = 0 if m == 1 else s
        rows.extend(r)
    n = len(shapes)
    flat = u32_array(rows, max(1, len(rows)))
    cshape = u32_array([])
    cstr = u32_array([], 3 * _abi.MAX_DIMS)
    k = lib().mtxc_pointwise_collapse(u32_array(out, max(rank, 1)), rank, flat, n, cshape, cstr)
    if k == UINT32_MAX:
        raise _abi.MtxcError(_abi.ERR_SHAPE, "pointwise output refused (rank or 32-bit size limit)")
    st = [list(cstr[i * _abi.MAX_DIMS:i * _abi.MAX_DIMS + k]) for i in range(n)]
    return PointwiseMeta(out, k, list(cshape[:k]), st, (cshape, cstr))


def pointwise(op: str, inputs, out: torch.Tensor | None = None, meta: PointwiseMeta | None = None) -> torch.Tensor:
    """greater / less / logical_and / where / floor / full / arctan2 / arcsin through mtxc_pointwise.  inputs
    are device tensors already in their common dtype (where: cond bool, then a and b; arctan2 / arcsin:
    float32, as the frontends cast them)."""
    import ctypes

    if meta is None:
        meta = pointwise_meta([list(t.shape) for t in inputs], [_check_strides(t) for t in inputs])
    data = inputs[-1]
    code = dtype_code(data.dtype)
    odt = (torch.bool if op in ("greater", "less", "logical_and") else
           torch.float32 if op in ("arctan2", "arcsin") else data.dtype)
    if out is None:
        out = torch.empty(meta.out_shape, dtype=odt, device=data.device)
    if out.numel() == 0:  # the reference's backends return before reading anything
        return out
    ptrs = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in inputs])
    cshape, cstr = meta.arrays
    check(lib().mtxc_pointwise(_abi.POINTWISE_OPS[op], code, out.data_ptr(), ptrs, len(inputs), meta.cdims, cshape,
                               cstr))
    return out


def arange(start: torch.Tensor, step: torch.Tensor, count: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """matrix::arange evaluated by mtxc_arange: count elements start + i * step; start and step are
    one-element device tensors of the output dtype (matrix::scalar(start, type), matrix::scalar(step, type))."""
    if start.dtype != step.dtype or start.numel() != 1 or step.numel() != 1:
        raise ValueError("arange: start and step are one element each of the output dtype")
    if out is None:
        out = torch.empty(count, dtype=start.dtype, device=start.device)
    check(lib().mtxc_arange(dtype_code(start.dtype), out.data_ptr(), start.data_ptr(), step.data_ptr(), count))
    return out


def softmax_lastdim(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's softmax trace over the last axis (max, sub, exp, sum, div) fused into one
    kernel (mtxc_softmax_lastdim).  x: contiguous rows of float32."""
    if x.dim() == 0 or x.stride(-1) != 1:
        raise ValueError("softmax_lastdim needs unit-stride rows")
    code = dtype_code(x.dtype)
    n = x.shape[-1]
    rows = x.numel() // n if n else 0
    row_stride = x.stride(-2) if x.dim() > 1 else n
    if x.dim() > 2 and not x.is_contiguous():
        raise ValueError("softmax_lastdim needs rows at a constant stride")
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    out_stride = out.stride(-2) if out.dim() > 1 else n
    check(lib().mtxc_softmax_lastdim(code, out.data_ptr(), x.data_ptr(), rows, n, row_stride, out_stride))
    return out


def reduce_pair(op: str, x: torch.Tensor, axis: int, keepdims: bool = False, meta: ReduceMeta | None = None):
    """(x.max(axis), x.argmax(axis)) -- or min / argmin -- from one read (mtxc_reduce_pair)."""
    code = dtype_code(x.dtype)
    if meta is None:
        meta = reduce_meta(list(x.shape), _check_strides(x), axis, keepdims)
    vals = torch.empty(meta.out_shape, dtype=x.dtype, device=x.device)
    idx = torch.empty(meta.out_shape, dtype=torch.int32, device=x.device)
    shape, s_out, s_in = meta.arrays
    check(lib().mtxc_reduce_pair(_abi.REDUCE_OPS[op], code, vals.data_ptr(), idx.data_ptr(), x.data_ptr(),
                                 meta.rstride & 0xFFFFFFFF, meta.rlen, meta.cdims, shape, s_out, s_in))
    return vals, idx


def reduce_sharded_launch(op: str, x_ptr: int, dtype: int, out_ptr: int, meta: ReduceMeta, offsets=None) -> None:
    """mtxc_reduce_sharded: this rank's slice of the reduced axis (`meta` describes it), the NCCL
    all-gather of every rank's partials and the ordered merge, on the thread's stream; needs the thread's
    communicator (shard.NativeComm).  offsets: the global index of each rank's first element (ArgMax /
    ArgMin)."""
    import ctypes

    shape, s_out, s_in = meta.arrays
    offs = (ctypes.c_int64 * len(offsets))(*[int(o) for o in offsets]) if offsets is not None else None
    check(lib().mtxc_reduce_sharded(_abi.REDUCE_OPS[op], dtype, out_ptr, x_ptr, meta.rstride & 0xFFFFFFFF, meta.rlen,
                                    meta.cdims, shape, s_out, s_in, offs))


def allreduce(op: str, buf: torch.Tensor) -> torch.Tensor:
    """In-place all-reduce (sum / max / min, rank-order merge) of a contiguous tensor across the
    communicator's ranks (mtxc_allreduce)."""
    if not buf.is_contiguous():
        raise ValueError("allreduce needs a contiguous tensor")
    check(lib().mtxc_allreduce(_abi.REDUCE_OPS[op], dtype_code(buf.dtype), buf.data_ptr(), buf.numel()))
    return buf


def merge_partials(op: str, values: torch.Tensor, indices: torch.Tensor | None = None, offsets=None):
    """Merges shard partials stacked on axis 0 ([parts, ...]) in shard order (mtxc_merge_partials).
    Returns the merged values (sum / max / min) or (values, global indices) (argmax / argmin)."""
    import ctypes

    parts = values.shape[0]
    outputs = values[0].numel()
    code = dtype_code(values.dtype)
    values = values.contiguous()
    if op in ("argmax", "argmin"):
        if indices is None or offsets is None:
            raise ValueError("argmax / argmin merges need the shards' indices and index offsets")
        indices = indices.contiguous()
        out_v = torch.empty(values.shape[1:], dtype=values.dtype, device=values.device)
        out_i = torch.empty(values.shape[1:], dtype=torch.int32, device=values.device)
        offs = (ctypes.c_int64 * parts)(*[int(o) for o in offsets])
        check(lib().mtxc_merge_partials(_abi.REDUCE_OPS[op], code, out_v.data_ptr(), out_i.data_ptr(),
                                        values.data_ptr(), indices.data_ptr(), offs, parts, outputs))
        return out_v, out_i
    out = torch.empty(values.shape[1:], dtype=values.dtype, device=values.device)
    check(lib().mtxc_merge_partials(_abi.REDUCE_OPS[op], code, out.data_ptr(), None, values.data_ptr(), None, None,
                                    parts, outputs))
    return out
