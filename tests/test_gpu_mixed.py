"""GPU parity for binary ops on operands of different dtypes, where the promotion is fused into the op
(mtxc_broadcast_binary_mixed: every pair of dtypes but Complex64).  The reference evaluates
astype(promote_types(a, b)) of the other operand and then the op; the oracle does exactly that, and the
fused kernel must give the same bits."""
import numpy as np
import pytest

from tests.helpers import assert_bits_equal
from tests.test_gpu_pointwise import dev
from tests.test_oracle_pin_pointwise import values

pytestmark = pytest.mark.gpu

OTHER = [1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12]  # every dtype but Float and Complex64
LAYOUTS = [([64, 1, 1024], [1, 16, 1024]), ([5], [3, 5]), ([7, 13], [7, 13]), ([4, 4096], [4096]), ([], [6])]


@pytest.mark.parametrize("code", OTHER)
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "equal"])
def test_mixed_float_and_other(gpu, port, code, op):
    rng = np.random.default_rng(400 + code)
    for sf, so in LAYOUTS:
        f = values(rng, 0, int(np.prod(sf)), special=True).reshape(sf)
        o = values(rng, code, int(np.prod(so)), special=code in (1, 10)).reshape(so)
        if op == "equal":  # make some pairs equal after the conversion
            fo = port.astype(o, np.float32, src_code=code, dst_code=0)
            k = min(f.size, fo.size) // 2
            f.reshape(-1)[:k] = fo.reshape(-1)[:k]
        o_as_f = port.astype(o, np.float32, src_code=code, dst_code=0)
        for a, b, ad, bd, tag in ((f, o_as_f, dev(f, 0), dev(o, code), "float op other"),
                                  (o_as_f, f, dev(o, code), dev(f, 0), "other op float")):
            want = port.binary(op, np.ascontiguousarray(a), np.ascontiguousarray(b))
            got = gpu.binary(op, ad, bd)
            gpu.sync()
            assert str(got.dtype) == "torch.float32"
            assert_bits_equal(got.cpu().numpy(), want, f"{tag}: {op} code {code} {sf} {so}")


def test_mixed_strided_and_transposed(gpu, port):
    import torch

    rng = np.random.default_rng(77)
    f = values(rng, 0, 40 * 33, special=True).reshape(40, 33)
    i = values(rng, 3, 33 * 40).reshape(33, 40)
    fd, idv = dev(f, 0), dev(i, 3)
    got = gpu.binary("mul", fd, idv.T)  # a transposed int32 operand
    gpu.sync()
    want = port.binary("mul", f, port.astype(i.T, np.float32, make_contig=False, src_code=3, dst_code=0))
    assert_bits_equal(got.cpu().numpy(), want, "mul f32 x int32^T")
    with pytest.raises(Exception):
        gpu.binary("max", fd, idv.T)  # max / min do not promote
    assert torch.cuda.is_available()


def _absorbing_pairs():
    """(result dtype D, other dtype S) with promote_types(D, S) == D, D not Float (covered above)."""
    from matrix_b200 import _abi

    from tests.test_oracle_pin_pointwise import ALL_CODES

    lib = _abi.lib()
    return [(d, s) for d in ALL_CODES for s in ALL_CODES
            if d != 0 and s != d and lib.mtxc_promote_types(d, s) == d]


def _safe(rng, code, n, nonzero):
    """Values of dtype `code` small enough that no op below overflows the promoted dtype, and nonzero
    where they divide (integer division by zero and INT_MIN / -1 are undefined in C++ and trap on x86)."""
    from tests.test_oracle_pin_pointwise import STORAGE

    if code == 7:
        return np.ones(n, dtype=np.bool_) if nonzero else rng.integers(0, 2, n).astype(np.bool_)
    if code in (1, 10):
        return values(rng, code, n)
    lo = -100 if np.issubdtype(STORAGE[code], np.signedinteger) else 0
    v = rng.integers(lo, 101, n)
    if nonzero:
        v[v == 0] = 7
    return v.astype(STORAGE[code])


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "equal"])
def test_mixed_result_of_one_operand(gpu, port, op):
    """Every pair of operand dtypes whose promoted dtype is one of the two, other than Float (Int64 with
    Int32 and the narrower integers, Int32 with Int16 / UInt32 / ..., a half type with Bool, ...): the
    fused kernel against the reference's evaluation (astype of the other operand, then the op in the
    result dtype), both operand orders, bit for bit."""
    import torch

    from matrix_b200.backend import CODE_TO_TORCH

    pairs = _absorbing_pairs()
    assert len(pairs) == 29
    rng = np.random.default_rng(500)
    for d, s in pairs:
        for sd, ss in (([64, 1, 96], [1, 16, 96]), ([7, 13], [7, 13]), ([], [5])):
            for d_first in (True, False):
                # the divisor (second operand) must stay nonzero after the conversion
                xd = _safe(rng, d, int(np.prod(sd)), nonzero=op == "div" and not d_first).reshape(sd)
                xs = _safe(rng, s, int(np.prod(ss)), nonzero=op == "div" and d_first).reshape(ss)
                xs_as_d = port.astype(xs, xd.dtype, src_code=s, dst_code=d)
                if d_first:
                    a, b, ad, bd = xd, xs_as_d, dev(xd, d), dev(xs, s)
                else:
                    a, b, ad, bd = xs_as_d, xd, dev(xs, s), dev(xd, d)
                want = port.binary(op, np.ascontiguousarray(a), np.ascontiguousarray(b), dtype_code=d)
                got = gpu.binary(op, ad, bd)
                gpu.sync()
                tag = f"{op} D={d} S={s} {'D op S' if d_first else 'S op D'} {sd} {ss}"
                assert got.dtype == CODE_TO_TORCH[d], tag
                g = got.cpu().numpy() if d != 10 else got.view(torch.uint16).cpu().numpy()
                if d == 10:  # BFloat16 bits as float32, so that NaNs (0 / 0) compare as NaNs
                    g, want = _bf16_as_f32(g), _bf16_as_f32(want)
                assert_bits_equal(g, want, tag)


def _bf16_as_f32(bits):
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


def _third_dtype_pairs():
    """(a dtype, b dtype, promoted dtype) with the promoted dtype neither operand's, both orders."""
    from matrix_b200 import _abi

    from tests.test_oracle_pin_pointwise import ALL_CODES

    lib = _abi.lib()
    return [(a, b, lib.mtxc_promote_types(a, b)) for a in ALL_CODES for b in ALL_CODES
            if a != b and lib.mtxc_promote_types(a, b) not in (a, b)]


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "equal"])
def test_mixed_third_dtype(gpu, port, op):
    """Every pair of operand dtypes that promotes to a third dtype (Float16 with Int32 -> Float, UInt8
    with Int8 -> Int16, Int16 with UInt32 -> Int32, ...), both orders: the fused kernel, which converts
    both operands as it reads them, against the reference's evaluation (astype of both, then the op),
    bit for bit."""
    from matrix_b200.backend import CODE_TO_TORCH
    from tests.test_oracle_pin_pointwise import STORAGE

    pairs = _third_dtype_pairs()
    assert len(pairs) == 52
    rng = np.random.default_rng(600)
    for ca, cb, d in pairs:
        for sa, sb in (([64, 1, 96], [1, 16, 96]), ([7, 13], [7, 13]), ([], [5])):
            xa = _safe(rng, ca, int(np.prod(sa)), nonzero=False).reshape(sa)
            xb = _safe(rng, cb, int(np.prod(sb)), nonzero=op == "div").reshape(sb)
            a_d = port.astype(xa, STORAGE[d], src_code=ca, dst_code=d)
            b_d = port.astype(xb, STORAGE[d], src_code=cb, dst_code=d)
            want = port.binary(op, np.ascontiguousarray(a_d), np.ascontiguousarray(b_d), dtype_code=d)
            got = gpu.binary(op, dev(xa, ca), dev(xb, cb))
            gpu.sync()
            tag = f"{op} {ca} with {cb} -> {d} {sa} {sb}"
            assert got.dtype == CODE_TO_TORCH[d], tag
            assert_bits_equal(got.cpu().numpy(), want, tag)


def test_mixed_entry_refusals(gpu):
    """mtxc_broadcast_binary_mixed refuses Complex64 operands, operands of one dtype, and a result dtype
    other than promote_types(a, b)."""
    import ctypes as C

    import torch

    from matrix_b200 import _abi

    lib = _abi.lib()
    a = torch.ones(8, dtype=torch.float16, device="cuda")
    b = torch.ones(8, dtype=torch.int32, device="cuda")
    out = torch.empty(8, dtype=torch.float32, device="cuda")
    u = _abi.u32_array

    def call(dtype, ca, cb):
        return lib.mtxc_broadcast_binary_mixed(0, dtype, ca, cb, C.c_void_p(out.data_ptr()),
                                               C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), 1, u([8]),
                                               u([1]), u([1]), u([1]))

    assert call(9, 9, 3) == _abi.ERR_UNSUPPORTED_DTYPE  # Complex64
    assert call(1, 1, 1) == _abi.ERR_INVALID_ARGUMENT  # one dtype
    assert call(1, 1, 3) == _abi.ERR_INVALID_ARGUMENT  # Float16 with Int32 is Float, not Float16
    assert call(0, 1, 3) == _abi.OK
    gpu.sync()
    assert bool((out == 2).all())
