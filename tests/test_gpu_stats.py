"""GPU parity for the fused mean / rms / norm (mtxc_reduce_stat) against the reference's composition
(mul, sum, astype, scalar division, sqrt) evaluated by the oracle.

Integer and Bool inputs are bit-exact (their sums wrap, so order does not matter).  Float inputs
differ only by the order of the additions (fp32 tree on the GPU, sequential in the input dtype on
the CPU): the result must be within tol of the CPU's, or -- where the CPU's sequential sum is itself
far from the exact sum (long runs, half-precision sums that stop growing) -- within tol of the
exact statistic computed in fp64 and no further from the CPU than the CPU is from exact.
tol = rtol * (sum|x| / n for a mean, |result| for rms / norm) + 2 ulp of the output dtype, with rtol
1e-5 (Float), 2^-10 (Float16), 2^-7 (BFloat16).
"""
import numpy as np
import pytest

from tests.helpers import assert_bits_equal
from tests.test_gpu_pointwise import comparable, dev, host
from tests.test_oracle_pin_pointwise import ALL_CODES, values

pytestmark = pytest.mark.gpu

RTOL = {0: 1e-5, 1: 2.0 ** -10, 10: 2.0 ** -7}
EPS_OUT = {0: 2.0 ** -23, 1: 2.0 ** -10, 10: 2.0 ** -7}


def as_f64(a, code):
    return comparable(np.asarray(a), code).astype(np.float64)


def exact_stat(kind, x64, axis, keep):
    if kind == "mean":
        return x64.mean(axis=axis, keepdims=keep)
    s = (x64 * x64).sum(axis=axis, keepdims=keep)
    return np.sqrt(s / x64.shape[axis]) if kind == "rms" else np.sqrt(s)


def check_float(kind, g, c, x64, axis, keep, code, oc, what):
    e = exact_stat(kind, x64, axis, keep)
    if kind == "mean":
        scale = np.abs(x64).sum(axis=axis, keepdims=keep) / max(x64.shape[axis], 1)
    else:
        scale = np.abs(e)
    tol = RTOL[code] * scale + 2 * EPS_OUT[oc] * np.maximum(np.abs(c), np.abs(g)) + 1e-30
    with np.errstate(invalid="ignore"):
        near_cpu = np.abs(g - c) <= tol
        near_exact = (np.abs(g - e) <= tol) & (np.abs(g - c) <= np.abs(c - e) + tol)
        both_nan = np.isnan(g) & np.isnan(c)
        same = g == c  # includes equal infinities (a Float16 sum past 65504)
    ok = near_cpu | near_exact | both_nan | same
    assert ok.all(), f"{what}: {np.count_nonzero(~ok)} of {ok.size} outside tolerance"


CASES = [([64, 4096], [4096, 1], 1), ([4096, 64], [64, 1], 0), ([2, 1 << 20], [1 << 20, 1], 1),
         ([40, 33], [1, 40], 1), ([8, 513, 129], [513 * 129, 129, 1], 1), ([7, 300], [300, 1], 1),
         ([3, 0], [1, 1], 1), ([1, 70000], [70000, 1], 1)]


@pytest.mark.parametrize("code", ALL_CODES)
@pytest.mark.parametrize("kind", ["mean", "rms", "norm"])
def test_stat(gpu, port, code, kind):
    import torch

    rng = np.random.default_rng(70 + code)
    for shape, strides, axis in CASES:
        need = sum((e - 1) * st for e, st in zip(shape, strides)) + 1 if all(shape) else 1
        base = values(rng, code, need, special=False)
        if code == 1:  # keep Float16 sums of squares mostly finite
            base = (base.astype(np.float32) / 16).astype(np.float16)
        xn = np.lib.stride_tricks.as_strided(base, shape, [st * base.itemsize for st in strides])
        xd = torch.as_strided(dev(base, code), shape, strides)
        for keep in (False, True):
            want, oc = port.stat(kind, xn, axis, keep, dtype_code=code)
            got = gpu.stat(kind, xd, axis, keep)
            gpu.sync()
            g = host(got, oc)
            assert g.shape == np.asarray(want).shape
            what = f"{kind} code {code} {shape}/{strides} axis {axis} keep {keep}"
            if code in (0, 1, 10):
                check_float(kind, as_f64(g, oc), as_f64(want, oc), as_f64(xn, code), axis, keep, code, oc, what)
            else:
                assert_bits_equal(comparable(g, oc), comparable(np.asarray(want), oc), what)
