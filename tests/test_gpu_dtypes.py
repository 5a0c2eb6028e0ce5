"""GPU parity for the half-precision and Bool dtypes (reference codes Float16 = 1, BFloat16 = 10,
Bool = 7).

* Max / Min / ArgMax / ArgMin are selections: bit-exact (all NaNs equal), with the same first-index
  and NaN rules as for float.
* Add / Sub / Mul / Div / Max / Min: bit-exact.  The GPU computes each half-precision op in fp32 and
  rounds once, which is exactly the correctly rounded half-precision result (fp32 has more than 2p + 2
  significand bits), and the reference's CPU arithmetic is correctly rounded too.
* Bool follows C++ bool arithmetic: the int result converted back to bool (a sum is a logical or).
* Half-precision sums: the reference accumulates sequentially in the half type itself, rounding every
  partial sum, while the GPU accumulates in fp32 and rounds once.  The GPU result must be within
  tol = 2^-10 * sum|x| (Float16) or 2^-7 * sum|x| (BFloat16) of the CPU result or of the exact sum.

numpy has no bfloat16: BFloat16 data travels as uint16 bits, with the dtype code given explicitly.
"""
import numpy as np
import pytest

from tests.helpers import assert_bits_equal, device_view, strided_view

pytestmark = pytest.mark.gpu

REDUCE_OPS = ["sum", "max", "min", "argmax", "argmin"]
BINARY_OPS = ["add", "sub", "mul", "div", "max", "min"]
KINDS = ["f16", "bf16", "bool"]
HALF_TOL = {"f16": 2.0 ** -10, "bf16": 2.0 ** -7}


def to_bf16_bits(x32: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even (NaN kept quiet)."""
    u = x32.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(x32)] = 0x7FC0
    return r


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def make(kind, rng, n, special=False):
    if kind == "bool":
        return rng.integers(0, 2, n).astype(np.bool_)
    v = (np.floor(rng.standard_normal(n) * 16) / 16).astype(np.float32)  # ties
    if special:
        pick = rng.integers(0, 12, n)
        v[pick == 0] = np.nan
        v[pick == 1] = np.inf
        v[pick == 2] = -np.inf
        v[pick == 3] = 0.0
        v[pick == 4] = -0.0
    return v.astype(np.float16) if kind == "f16" else to_bf16_bits(v)


def code(kind):
    return {"f16": 1, "bf16": 10, "bool": 7}[kind]


def to_torch(kind, base):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(base)).cuda()
    return t.view(torch.bfloat16) if kind == "bf16" else t


def host_bits(kind, t):
    import torch

    if kind == "bf16" and t.dtype == torch.bfloat16:
        return t.view(torch.uint16).cpu().numpy()
    return t.cpu().numpy()


def as_f64(kind, a):
    return bf16_to_f32(a).astype(np.float64) if kind == "bf16" else a.astype(np.float64)


def check_reduce(gpu, port, kind, op, base, shape, strides, off, axis):
    x = strided_view(base, shape, strides, off)
    cpu = port.reduce(op, x, axis, False, dtype_code=code(kind))
    xd = device_view(to_torch(kind, base), shape, strides, off)
    out = gpu.reduce(op, xd, axis)
    gpu.sync()
    g = host_bits(kind, out)
    tag = f"{kind} {op} {shape}/{strides}+{off} axis {axis}"
    if op == "sum" and kind != "bool":
        gf, cf = as_f64(kind, g), as_f64(kind, cpu)
        xf = as_f64(kind, np.ascontiguousarray(x))
        tol = HALF_TOL[kind] * np.abs(xf).sum(axis) + 1e-30
        exact = xf.sum(axis)
        with np.errstate(invalid="ignore"):
            ok = (np.abs(gf - cf) <= tol) | (np.abs(gf - exact) <= tol) | (np.isnan(gf) & np.isnan(cf))
        assert ok.all(), f"{tag}: {np.count_nonzero(~ok)} sums outside tolerance"
    else:
        if kind == "bf16" and op in ("max", "min"):
            g, cpu = bf16_to_f32(g), bf16_to_f32(cpu)  # compare NaNs as NaNs
        assert_bits_equal(g, cpu, tag)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("op", REDUCE_OPS)
def test_reduce_half_and_bool(gpu, port, kind, op):
    rng = np.random.default_rng(17)
    cases = [([7, 300], [300, 1], 0), ([33, 1000], [1000, 1], 0), ([4, 70000], [70000, 1], 0),
             ([8, 513, 129], [513 * 129, 129, 1], 0), ([16, 64, 512], [64 * 512, 512, 1], 0),
             ([50, 64], [1, 50], 0), ([40, 33], [40, 1], 3), ([3, 1 << 17], [1 << 17, 1], 0)]
    for shape, strides, off in cases:
        need = off + sum((e - 1) * s for e, s in zip(shape, strides)) + 1
        base = make(kind, rng, need, special=(op != "sum"))
        for axis in range(len(shape)):
            check_reduce(gpu, port, kind, op, base, shape, strides, off, axis)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("op", BINARY_OPS)
def test_broadcast_half_and_bool(gpu, port, kind, op):
    rng = np.random.default_rng(23)
    for sa, sb in (([8, 1, 64], [1, 16, 64]), ([5], [3, 5]), ([7, 13], [7, 13]), ([6, 1, 1, 8], [1, 5, 7, 8]),
                   ([64, 1024], [64, 1])):
        a = make(kind, rng, int(np.prod(sa)), special=True).reshape(sa)
        b = make(kind, rng, int(np.prod(sb)), special=True).reshape(sb)
        if kind == "bool" and op == "div":
            b = np.ones_like(b)  # bool division by false is undefined (a trap on x86)
        cpu = port.binary(op, a, b, dtype_code=code(kind))
        out = gpu.binary(op, to_torch(kind, a), to_torch(kind, b))
        gpu.sync()
        g = host_bits(kind, out)
        if kind == "bf16":
            g, cpu = bf16_to_f32(g), bf16_to_f32(cpu)
        assert_bits_equal(g, cpu, f"{kind} {op} {sa} {sb}")


@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_reduce_pair_half(gpu, port, kind):
    rng = np.random.default_rng(29)
    shape = [16, 2048, 256]
    base = make(kind, rng, int(np.prod(shape)), special=True)
    xd = to_torch(kind, base).reshape(shape)
    v, i = gpu.reduce_pair("max", xd, 1)
    gpu.sync()
    x = base.reshape(shape)
    want_v = port.reduce("max", x, 1, dtype_code=code(kind))
    gv = host_bits(kind, v)
    if kind == "bf16":
        gv, want_v = bf16_to_f32(gv), bf16_to_f32(want_v)
    assert_bits_equal(gv, want_v, "pair value")
    assert_bits_equal(i.cpu().numpy(), port.reduce("argmax", x, 1, dtype_code=code(kind)), "pair index")


@pytest.mark.parametrize("kind", ["f16", "bf16"])
@pytest.mark.parametrize("op", ["max", "min", "argmax", "argmin"])
def test_reduce_half_packed(gpu, port, kind, op):
    """The packed (value, index) fold of the half types (16-byte lanes of 8 elements compared as the
    floats they widen to), over columns and over rows: NaN, infinities, +-0 and ties; values rising or
    falling along the reduced axis (a new best every row); the 4-byte fallback lanes and misaligned
    operands; chunks of 1 and 3 rows as well as the default, so the 16-bit chunk numbers turn into
    indices mid-run.  Bit-exact."""
    import ctypes

    from matrix_b200 import _abi

    set_chunk = _abi.lib().mtxc_debug_set_col_chunk
    set_chunk.argtypes, set_chunk.restype = [ctypes.c_uint32], ctypes.c_uint32
    rng = np.random.default_rng(31)
    cases = [([300, 64], 0, 0), ([3, 257, 48], 1, 0), ([1000, 20], 0, 0), ([700, 96], 0, 4),
             ([64, 3000], 1, 0), ([8, 70001], 1, 0), ([5, 4099], 1, 3)]  # the last three: over rows
    for chunk in (65535, 1, 3):
        set_chunk(chunk)
        try:
            for shape, axis, off in cases:
                strides = [int(np.prod(shape[i + 1:])) for i in range(len(shape))]
                n = int(np.prod(shape))
                for pattern in ("special", "rising", "falling"):
                    if pattern == "special":
                        v = make(kind, rng, n, special=True)
                    else:
                        ramp = (np.indices(shape)[axis].reshape(-1) / 32.0 - 4.0).astype(np.float32)
                        ramp = ramp if pattern == "rising" else -ramp
                        v = ramp.astype(np.float16) if kind == "f16" else to_bf16_bits(ramp)
                    base = np.concatenate([np.zeros(off, dtype=v.dtype), v])
                    check_reduce(gpu, port, kind, op, base, shape, strides, off, axis)
        finally:
            set_chunk(65535)
