"""GPU parity for astype / copy, exp and sqrt on Float16, equal, and the make_pointwise family
(greater, less, logical_and, where, floor, full), through the C ABI, against the oracle.

All of these are bit-exact (NaNs compared as NaNs) except Float16 exp, which is CUDA's expf rounded
once to half against glibc's expf rounded once: within 1 half-precision ulp.  Shapes cover both
kernels: rows whose innermost axis allows 16-byte chunks (with inputs broadcast along the row) and
the generic strided decode (transposes, odd lengths, offsets), plus empty and single-element cases.
Float-to-integer conversions use values inside the destination's range (outside it C++ leaves the
conversion undefined, so the reference has no single answer).
"""
import numpy as np
import pytest

from tests.helpers import assert_bits_equal, ulp_distance
from tests.test_oracle_pin_pointwise import ALL_CODES, INT_RANGE, STORAGE, values

pytestmark = pytest.mark.gpu


def torch_dtype(code):
    import torch

    return {0: torch.float32, 1: torch.float16, 2: torch.uint8, 3: torch.int32, 4: torch.int16, 5: torch.uint32,
            6: torch.uint16, 7: torch.bool, 8: torch.int8, 10: torch.bfloat16, 11: torch.int64,
            12: torch.uint64}[code]


def dev(a: np.ndarray, code):
    """numpy storage -> device tensor of dtype `code`, keeping the view's shape and strides."""
    import torch

    base = np.array(a, order="C", copy=True)  # (np.ascontiguousarray would make a 0-d array 1-d)
    t = torch.from_numpy(base).cuda()
    return t.view(torch.bfloat16) if code == 10 else t


def host(t, code):
    import torch

    if code == 10:
        return t.contiguous().view(torch.uint16).cpu().numpy()
    return t.contiguous().cpu().numpy()


def comparable(a: np.ndarray, code):
    """Values for comparison: BFloat16 bits widened to float32 so NaNs compare as NaNs."""
    if code == 10:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a


def views(rng, code, dst=None):
    """(numpy view, device view) pairs over one base: contiguous long rows, a transpose, a column
    slice with an offset, a broadcast (stride-0) axis, odd lengths, one element, an empty one."""
    import torch

    out = []
    for shape in ([64, 4096], [3, 5, 7], [1000], [1], [0, 5]):
        n = int(np.prod(shape))
        base = values(rng, code, max(n, 1), dst_code=dst, special=dst not in INT_RANGE)
        x = base[:n].reshape(shape)
        out.append((x, dev(x, code)))
    base = values(rng, code, 33 * 40, dst_code=dst, special=dst not in INT_RANGE).reshape(33, 40)
    d = dev(base, code)
    out.append((base.T, d.T))
    out.append((base[:, 3:35], d[:, 3:35]))
    row = values(rng, code, 256, dst_code=dst, special=dst not in INT_RANGE)
    out.append((np.broadcast_to(row, (48, 256)), dev(row, code).expand(48, 256)))
    return out


@pytest.mark.parametrize("src", ALL_CODES)
def test_astype_all_pairs(gpu, port, src):
    rng = np.random.default_rng(300 + src)
    for dst in ALL_CODES:
        for xn, xd in views(rng, src, dst):
            for mc in (True, False):
                want = port.astype(xn, STORAGE[dst], make_contig=mc, src_code=src, dst_code=dst)
                got = gpu.astype(xd, torch_dtype(dst), make_contig=mc)
                gpu.sync()
                assert_bits_equal(comparable(host(got, dst), dst), comparable(np.ascontiguousarray(want), dst),
                                  f"astype {src}->{dst} {xn.shape}/{xn.strides} contig={mc}")


def test_astype_rounding_boundaries(gpu, port):
    """Integers whose conversion to float / bfloat16 rounds at a tie after a first rounding (a float
    intermediate would round twice), and half <-> bfloat16 through float."""
    ints = np.array([16842753, -16842753, 16777217, 2**31 - 1, -2**31, 33554435, 65520, 65519, 2049],
                    dtype=np.int32)
    i64 = np.array([(1 << 40) + (1 << 32) + 1, -(1 << 62) - (1 << 54) - 1, 2**63 - 1, 9007199791611905],
                   dtype=np.int64)
    u64 = np.array([(1 << 63) + (1 << 55) + 1, 2**64 - 1, 0x8000008000000001], dtype=np.uint64)
    for x, src in ((ints, 3), (i64, 11), (u64, 12)):
        for dst in (0, 1, 10):
            want = port.astype(x, STORAGE[dst], src_code=src, dst_code=dst)
            got = gpu.astype(dev(x, src), torch_dtype(dst))
            gpu.sync()
            assert_bits_equal(comparable(host(got, dst), dst), comparable(want, dst), f"{src}->{dst}")


def test_sqrt_and_exp_float16(gpu, port):
    import torch

    rng = np.random.default_rng(31)
    for dt, code in ((np.float32, 0), (np.float16, 1)):
        x = np.abs(rng.standard_normal(64 * 1024) * 30).astype(dt)
        x[::97] = np.array(np.nan, dtype=dt)
        x[1::89] = np.array(np.inf, dtype=dt)
        x[2::83] = 0
        for xn, xd in ((x.reshape(64, 1024), dev(x, code).reshape(64, 1024)),
                       (x.reshape(64, 1024)[:, 5:900:3], dev(x, code).reshape(64, 1024)[:, 5:900:3])):
            got = gpu.unary("sqrt", xd)
            gpu.sync()
            assert_bits_equal(got.cpu().numpy(), port.unary("sqrt", xn), f"sqrt {dt}")
        if code == 1:
            y = (rng.standard_normal(64 * 1024) * 4).astype(np.float16)
            got = gpu.unary("exp", dev(y, 1)).cpu().numpy()
            gpu.sync()
            want = port.unary("exp", y)
            fin = np.isfinite(want) & np.isfinite(got)
            assert (np.isfinite(want) == np.isfinite(got)).all()
            assert ulp_distance(got[fin], want[fin]).max() <= 1
    with pytest.raises(Exception):
        gpu.unary("sqrt", dev(np.ones(16, dtype=np.int32), 3))
    assert torch.cuda.is_available()


@pytest.mark.parametrize("code", ALL_CODES)
def test_equal(gpu, port, code):
    rng = np.random.default_rng(41 + code)
    for sa, sb in (([8, 1, 4096], [1, 16, 4096]), ([5], [3, 5]), ([7, 13], [7, 13]), ([6, 1, 1, 8], [1, 5, 7, 8]),
                   ([64, 1024], [64, 1]), ([], [4])):
        a = values(rng, code, int(np.prod(sa)), special=True).reshape(sa)
        b = values(rng, code, int(np.prod(sb)), special=True).reshape(sb)
        fb, fa = b.reshape(-1), a.reshape(-1)
        k = min(fa.size, fb.size) // 2
        fb[:k] = fa[:k]
        want = port.binary("equal", a, b, dtype_code=code)
        got = gpu.binary("equal", dev(a, code), dev(b, code))
        gpu.sync()
        assert_bits_equal(comparable(host(got, code), code), comparable(want, code), f"equal {code} {sa} {sb}")


@pytest.mark.parametrize("code", ALL_CODES)
def test_pointwise_family(gpu, port, code):
    rng = np.random.default_rng(51 + code)
    shapes = [([64, 4096], [4096], [64, 1]), ([3, 1, 5], [4, 5], [3, 4, 1]), ([1000], [1], [1000]),
              ([2, 3, 4, 5], [1, 3, 1, 5], [5]), ([0, 3], [3], [1, 3]), ([], [], [])]
    for s0, s1, s2 in shapes:
        a = values(rng, code, int(np.prod(s0)), special=True).reshape(s0)
        b = values(rng, code, int(np.prod(s1)), special=True).reshape(s1)
        c = values(rng, code, int(np.prod(s2)), special=True).reshape(s2)
        cond = rng.integers(0, 2, int(np.prod(s2))).astype(np.bool_).reshape(s2)
        at = dev(a, code)
        # a transposed view of `a` exercises the generic decode with the same values
        aT, atT = (a.T, at.mT) if a.ndim == 2 else (a, at)
        d = values(rng, code, int(np.prod(s0)), special=True).reshape(aT.shape)
        cases = [("greater", [a, b]), ("less", [aT, d]), ("where", [cond, a, c]), ("floor", [aT]), ("full", [b])]
        if code == 7:
            cases.append(("logical_and", [a, c]))
        for op, ins in cases:
            dins = []
            for x in ins:
                if x is aT:
                    dins.append(atT)
                elif x.dtype == np.bool_ and op == "where" and x is cond:
                    dins.append(dev(x, 7))
                else:
                    dins.append(dev(x, code))
            want = port.pointwise(op, ins, dtype_code=code)
            got = gpu.pointwise(op, dins)
            gpu.sync()
            oc = 7 if op in ("greater", "less", "logical_and") else code
            assert_bits_equal(comparable(host(got, oc), oc), comparable(want, oc),
                              f"{op} {code} {[x.shape for x in ins]}")


def test_pointwise_errors(gpu):
    import torch

    from matrix_b200 import _abi

    x = torch.zeros(8, dtype=torch.int32, device="cuda")
    with pytest.raises(_abi.MtxcError) as e:
        gpu.pointwise("logical_and", [x, x])
    assert e.value.code == _abi.ERR_UNSUPPORTED_DTYPE
    with pytest.raises(_abi.MtxcError):
        gpu.astype(torch.zeros(4, dtype=torch.complex64, device="cuda"), torch.float32)


ATAN2_ASIN_ULP = 3  # CUDA's atan2f / asinf against glibc's float atan2 / asin (the oracle's std:: calls)


def _on_device(view: np.ndarray, base: np.ndarray, base_dev):
    """The device tensor with `view`'s shape, strides and offset over base_dev (a copy of base)."""
    import torch

    off = (view.__array_interface__["data"][0] - base.__array_interface__["data"][0]) // view.itemsize
    return torch.as_strided(base_dev, view.shape, [st // view.itemsize for st in view.strides], off)


def test_arctan2_and_arcsin(gpu, port):
    """arctan2 / arcsin (Float inputs, as the frontends cast them; Matrix.mm:13573-13580): CUDA's atan2f /
    asinf against the CPU backends' std::atan2 / std::asin, within ATAN2_ASIN_ULP ulp, NaN where the CPU has
    NaN.  Special values: signed zeros, infinities, NaN, |x| > 1.  Row-broadcast, strided, transposed and
    single-element layouts."""
    import torch

    rng = np.random.default_rng(31)
    a = (rng.standard_normal((257, 1024)) * 5).astype(np.float32)
    b = (rng.standard_normal((1024,)) * 5).astype(np.float32)
    a[0, :10] = [0.0, -0.0, 0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, np.inf, -1e-30]
    b[:10] = [0.0, 0.0, -0.0, -0.0, np.inf, np.inf, 1.0, np.nan, -np.inf, 1e-30]
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    cases = [((a, a, ad), (b, b, bd)), ((a[:, ::3], a, ad), (b[::3], b, bd)),
             ((a.T[:7], a, ad), (a.T[7:14], a, ad)), ((a[:1, :1], a, ad), (b[:1], b, bd))]
    for (x, xb, xbd), (y, yb, ybd) in cases:
        got = gpu.pointwise("arctan2", [_on_device(x, xb, xbd), _on_device(y, yb, ybd)])
        gpu.sync()
        want = port.pointwise("arctan2", [x, y])
        g = got.cpu().numpy()
        assert g.shape == want.shape
        assert ulp_distance(g, want).max() <= ATAN2_ASIN_ULP, "arctan2 beyond the ulp bound"
        assert np.array_equal(np.isnan(g), np.isnan(want))
    x = rng.uniform(-1.25, 1.25, (513, 777)).astype(np.float32)
    x[0, :8] = [1.0, -1.0, 0.0, -0.0, np.nan, np.inf, 1.0000001, -0.9999999]
    xd = torch.from_numpy(x).cuda()
    for v in (x, x[:, 1::2], x[5]):
        got = gpu.pointwise("arcsin", [_on_device(v, x, xd)]).cpu().numpy()
        want = port.pointwise("arcsin", [v])
        assert ulp_distance(got, want).max() <= ATAN2_ASIN_ULP, "arcsin beyond the ulp bound"
        assert np.array_equal(np.isnan(got), np.isnan(want))
        zero = (got == 0) & (want == 0)
        assert np.array_equal(np.signbit(got[zero]), np.signbit(want[zero]))


@pytest.mark.parametrize("code", [c for c in ALL_CODES if c != 7])
def test_arange(gpu, port, code):
    """arange (Matrix.mm:13595-13604, backend 14167-14180): bit-exact against the oracle for every dtype
    but Bool, incl. negative and fractional steps, wrapping integers, float rounding past 2^24 elements, an
    empty and a one-element range, and an output that is not 16-byte aligned."""
    import torch

    from matrix_b200 import _abi
    from tests.test_oracle_pin_pointwise import bf16_bits

    def scalars(start, step):
        if code in (0, 1, 10):
            s32 = np.array([start, step], dtype=np.float32)
            if code == 0:
                return s32
            if code == 1:
                return s32.astype(np.float16)
            return bf16_bits(s32)
        return np.array([int(start), int(step)], dtype=np.int64).astype(STORAGE[code])

    cases = [(0, 1, 0), (0, 1, 1), (3, 2, 1000), (-7, 3, 4099), (100, -1, 300), (0.5, 0.25, 70000),
             (-1e3, 0.1, 20001), (1, 7, (1 << 25) + 3)]
    for start, step, n in cases:
        sv = scalars(start, step)
        want = port.arange(sv[0], sv[1], n, STORAGE[code], dtype_code=code)
        st = dev(sv, code)
        for offset in (0, 1):
            out = torch.empty(n + offset, dtype=torch_dtype(code), device="cuda")[offset:]
            gpu.arange(st[0:1], st[1:2], n, out=out)
            gpu.sync()
            assert_bits_equal(comparable(host(out, code), code), comparable(want, code),
                              f"arange {code} {start} {step} {n} offset {offset}")
    b = torch.ones(2, dtype=torch.bool, device="cuda")
    with pytest.raises(_abi.MtxcError) as e:
        gpu.arange(b[0:1], b[1:2], 4)
    assert e.value.code == _abi.ERR_UNSUPPORTED_DTYPE
