"""GPU parity of the broadcasted binary ops and exp against the CPU oracle.

``a <op> b`` goes through mtxc_broadcast_binary with the metadata the reference's operator
builds (broadcast_shapes + collapse_dims over result / a / b strides).  Every element must be
bit-identical with the reference CPU loop: each is a single IEEE-rounded operation (or a
std::max / std::min selection).  exp is compared in ulp.
"""
import numpy as np
import pytest

from tests.helpers import (EXP_ULP, INT_DTYPES, assert_bits_equal, device_view, make_values, strided_view, to_device,
                           ulp_distance)

pytestmark = pytest.mark.gpu

OPS = ["add", "sub", "mul", "div", "max", "min"]


def contiguous_strides(shape):
    return [int(np.prod(shape[i + 1:])) for i in range(len(shape))]


def check_binary(backend, port, op, a_base, a_shape, a_strides, a_off, b_base, b_shape, b_strides, b_off, what=""):
    a = strided_view(a_base, a_shape, a_strides, a_off)
    b = strided_view(b_base, b_shape, b_strides, b_off)
    cpu = port.binary(op, a, b)
    ad = device_view(to_device(a_base), a_shape, a_strides, a_off)
    bd = device_view(to_device(b_base), b_shape, b_strides, b_off)
    out = backend.binary(op, ad, bd)
    backend.sync()
    assert_bits_equal(out.cpu().numpy(), cpu, f"{what} {op} {a_shape}/{a_strides}+{a_off} {b_shape}/{b_strides}+{b_off} "
                                              f"{a_base.dtype}")


def operands(rng, dtype, na, nb, op, kind="uniform"):
    a = make_values(rng, na, dtype, kind if np.dtype(dtype) == np.float32 else "full")
    b = make_values(rng, nb, dtype, kind if np.dtype(dtype) == np.float32 else "full")
    if op == "div" and np.dtype(dtype).kind in "iu":
        b[b == 0] = 1  # integer division by zero is undefined in the reference (a trap on x86)
        if np.dtype(dtype).kind == "i":
            b[b == -1] = 3  # INT_MIN / -1 traps as well
    return a, b


PAIRS = [
    ([8, 1, 64], [1, 16, 64]),      # C2 in miniature
    ([5], [3, 5]),                  # rank mismatch
    ([3, 1], [1, 4]),
    ([1], [4, 4]),
    ([4, 4], [1]),
    ([7, 13], [7, 13]),             # no broadcast, odd inner extent
    ([2, 3, 1, 5], [3, 4, 1]),
    ([6, 1, 1, 8], [1, 5, 7, 8]),
    ([2, 1, 3, 1, 4, 1], [1, 5, 1, 6, 1, 7]),
    ([64, 1024], [1024]),           # row vector
    ([64, 1024], [64, 1]),          # column vector
    ([1, 1, 4096], [3, 2, 4096]),
    ([33, 1, 40], [1, 17, 40]),
]


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("pair", PAIRS, ids=lambda p: f"{'x'.join(map(str, p[0]))}-{'x'.join(map(str, p[1]))}")
def test_binary_shapes_f32(gpu, port, op, pair):
    rng = np.random.default_rng(1)
    sa, sb = pair
    a, b = operands(rng, np.float32, int(np.prod(sa)), int(np.prod(sb)), op)
    check_binary(gpu, port, op, a, sa, contiguous_strides(sa), 0, b, sb, contiguous_strides(sb), 0)
    check_binary(gpu, port, op, b, sb, contiguous_strides(sb), 0, a, sa, contiguous_strides(sa), 0, "swapped")


@pytest.mark.parametrize("dtype", INT_DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("op", OPS)
def test_binary_int_dtypes(gpu, port, dtype, op):
    rng = np.random.default_rng(2)
    for sa, sb in ([[8, 1, 64], [1, 16, 64]], [[5], [3, 5]], [[7, 13], [7, 13]], [[6, 1, 1, 8], [1, 5, 7, 8]]):
        a, b = operands(rng, dtype, int(np.prod(sa)), int(np.prod(sb)), op)
        check_binary(gpu, port, op, a, sa, contiguous_strides(sa), 0, b, sb, contiguous_strides(sb), 0)


@pytest.mark.parametrize("op", OPS)
def test_binary_float_specials(gpu, port, op):
    """NaN / inf / signed zeros / extremes: IEEE results and std::max / std::min selection
    (the first operand is kept unless the second is strictly better; NaN compares false)."""
    rng = np.random.default_rng(3)
    a = make_values(rng, 40 * 256, np.float32, "special")
    b = make_values(rng, 40 * 256, np.float32, "special")
    check_binary(gpu, port, op, a, [40, 256], [256, 1], 0, b, [40, 256], [256, 1], 0)
    check_binary(gpu, port, op, a, [40, 1, 16], [16, 16, 1], 0, b, [1, 30, 16], [480, 16, 1], 0)
    denorm = (rng.standard_normal(4096) * 1e-39).astype(np.float32)
    check_binary(gpu, port, op, denorm, [4096], [1], 0, a[:4096].copy(), [4096], [1], 0, "denormals")


@pytest.mark.parametrize("op", ["add", "mul", "div", "max"])
def test_binary_strided_views(gpu, port, op):
    """Transposed, offset (unaligned) and expanded operands take the generic path."""
    rng = np.random.default_rng(4)
    a = make_values(rng, 1 << 16, np.float32, "uniform")
    b = make_values(rng, 1 << 16, np.float32, "uniform")
    cases = [
        (([64, 100], [1, 128], 0), ([64, 100], [100, 1], 0)),      # transposed a
        (([50, 64], [128, 1], 1), ([50, 64], [64, 1], 0)),         # unaligned a
        (([50, 64], [64, 1], 0), ([1, 64], [64, 1], 3)),           # unaligned broadcast b
        (([8, 16, 32], [0, 32, 1], 0), ([8, 16, 32], [512, 32, 1], 0)),  # expanded a
        (([10, 20, 30], [1, 10, 200], 0), ([30], [1], 5)),
    ]
    for (sa, ta, oa), (sb, tb, ob) in cases:
        check_binary(gpu, port, op, a, sa, ta, oa, b, sb, tb, ob)


def test_binary_scalar_and_empty(gpu, port):
    import torch

    rng = np.random.default_rng(5)
    a, b = operands(rng, np.float32, 1, 1, "add")
    for op in OPS:
        check_binary(gpu, port, op, a, [], [], 0, b, [], [], 0, "0-d")
    x = torch.empty((0, 4), device="cuda")
    y = torch.empty((1, 4), device="cuda")
    out = gpu.binary("add", x, y)
    gpu.sync()
    assert out.shape == (0, 4)
    with pytest.raises(ValueError):
        gpu.binary_meta([3, 4], [4, 1], [5, 4], [4, 1])


@pytest.mark.slow
def test_config2_add_mul_full(gpu, port):
    """C2: a[256,1,4096] (+, *) b[1,512,4096] -> [256,512,4096], bit-exact."""
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, 256 * 4096).astype(np.float32)
    b = rng.uniform(-1, 1, 512 * 4096).astype(np.float32)
    for op in ("add", "mul"):
        check_binary(gpu, port, op, a, [256, 1, 4096], [4096, 4096, 1], 0, b, [1, 512, 4096], [2097152, 4096, 1], 0,
                     "C2")


# ------------------------------------------------------------------------------------------
# exp
# ------------------------------------------------------------------------------------------
def check_exp(backend, port, base, shape, strides, off=0, what=""):
    x = strided_view(base, shape, strides, off)
    cpu = port.exp(x)
    xd = device_view(to_device(base), shape, strides, off)
    out = backend.exp(xd)
    backend.sync()
    g = out.cpu().numpy()
    assert g.shape == cpu.shape
    d = ulp_distance(g, cpu)
    assert d.max(initial=0) <= EXP_ULP, f"{what} exp {shape}: max ulp {d.max()} at {np.argmax(d)}"


def test_exp_shapes_and_specials(gpu, port):
    rng = np.random.default_rng(6)
    base = (rng.standard_normal(1 << 16) * 30).astype(np.float32)
    for shape, strides, off in (([1 << 16], [1], 0), ([64, 1024], [1024, 1], 0), ([64, 100], [1, 128], 0),
                                ([50, 64], [128, 1], 3), ([7, 9, 13], [117, 13, 1], 0), ([], [], 0)):
        check_exp(gpu, port, base, shape, strides, off)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 88.72, 88.73, -87.3, -103.0, -104.0, 1e-30, -1e-30]
                       * 4, dtype=np.float32)
    check_exp(gpu, port, special, [special.size], [1], 0, "special")


# ------------------------------------------------------------------------------------------
# softmax trace (C5a in miniature): max, sub, exp, sum, div
# ------------------------------------------------------------------------------------------
def test_softmax_trace_matches_oracle(gpu, port):
    import torch

    rng = np.random.default_rng(4)
    rows, cols = 64, 4096
    x = (rng.standard_normal(rows * cols) * 2).astype(np.float32).reshape(rows, cols)
    m = port.reduce("max", x, -1, True)
    e = port.exp(port.binary("sub", x, m))
    y_cpu = port.binary("div", e, port.reduce("sum", e, -1, True))

    xd = torch.from_numpy(x).cuda()
    md = gpu.reduce("max", xd, -1, True)
    ed = gpu.exp(gpu.binary("sub", xd, md))
    yd = gpu.binary("div", ed, gpu.reduce("sum", ed, -1, True))
    gpu.sync()
    y = yd.cpu().numpy()
    np.testing.assert_allclose(y, y_cpu, rtol=1e-5, atol=0)
    assert_bits_equal(md.cpu().numpy(), m, "softmax max")


def test_long_rows_are_segmented(gpu, port):
    """Fully collapsed contiguous operands form one long row, which the row kernels cut into
    segments; a column operand (inner stride 0) keeps the vector path."""
    rng = np.random.default_rng(8)
    n = 3 * (1 << 20) + 4 * 37  # several segments plus a partial one
    a = make_values(rng, n, np.float32, "uniform")
    b = make_values(rng, n, np.float32, "uniform")
    for op in ("add", "div"):
        check_binary(gpu, port, op, a, [n], [1], 0, b, [n], [1], 0, "one long row")
    col = make_values(rng, 96, np.float32, "uniform")
    big = make_values(rng, 96 * 70000, np.float32, "uniform")
    for op in ("sub", "div"):
        check_binary(gpu, port, op, big, [96, 70000], [70000, 1], 0, col, [96, 1], [1, 1], 0, "column operand")
        check_binary(gpu, port, op, col, [95, 1], [1, 1], 1, big, [95, 70000], [70000, 1], 0, "column first")
    check_exp(gpu, port, a, [n], [1], 0, "one long row")
    check_exp(gpu, port, big, [96, 70000], [70000, 1], 0, "rows")


GROUPED = [
    # (a shape, b shape): both contiguous along the row, exactly one broadcast along the next axis out
    ([4, 1, 64], [1, 13, 64]),      # a shared; 13 rows = one full group of 8 and a partial one
    ([1, 21, 32], [6, 1, 32]),      # b shared along the 21-axis (partial last group)
    ([2, 1, 20480], [1, 9, 20480]),  # rows of 5120 vectors: segmented, and a partial group
    ([3, 2, 1, 8], [1, 1, 16, 8]),  # several outer axes
    ([1, 8, 256], [5, 8, 256]),     # neither operand shared along the next axis out: the row kernel
]


@pytest.mark.parametrize("dtype", [np.float32, np.int32, np.uint8, np.float16], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("op", OPS)
def test_grouped_rows(gpu, port, dtype, op):
    """Layouts the grouped row kernel takes (rows sharing a broadcast operand, 8 per work unit; 2 for
    division), with partial last groups, the shared operand on either side and segmented rows."""
    rng = np.random.default_rng(91)
    for sa, sb in GROUPED:
        if np.dtype(dtype) == np.float16:
            a = (rng.standard_normal(int(np.prod(sa))) * 4).astype(np.float16)
            b = (rng.standard_normal(int(np.prod(sb))) * 4).astype(np.float16)
        else:
            a, b = operands(rng, dtype, int(np.prod(sa)), int(np.prod(sb)), op)
        if op == "div" and np.dtype(dtype).kind in "iu":  # a is the divisor of the swapped check
            a[a == 0] = 1
            if np.dtype(dtype).kind == "i":
                a[a == -1] = 3
        check_binary(gpu, port, op, a, sa, contiguous_strides(sa), 0, b, sb, contiguous_strides(sb), 0, "grouped")
        check_binary(gpu, port, op, b, sb, contiguous_strides(sb), 0, a, sa, contiguous_strides(sa), 0, "grouped swapped")
