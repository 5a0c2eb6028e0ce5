"""Shared helpers for the parity tests: seeded inputs, strided views on host and device, and
the comparison rules.

Comparison rules (stated once, used everywhere):
  * integer results, ArgMax / ArgMin indices, Max / Min values and every single elementwise
    float op (add, sub, mul, div, max, min) must match the oracle bit for bit, with one
    exception: all NaNs compare equal.  The sign and payload of a NaN that arithmetic creates
    (inf - inf, 0 * inf, ...) or propagates are architecture-defined -- x86 makes 0xffc00000,
    the reference's ARM host 0x7fc00000, NVIDIA GPUs 0x7fffffff -- so they carry no meaning;
  * float sums, whose summation order differs from the reference's sequential loop, must satisfy
    |gpu - cpu| <= tol with tol = 1e-5 * sum(|x|) over the reduced run (plus 1e-30).  Where the
    reference's own sequential fp32 sum is off the exact (fp64) sum by more than tol -- long runs
    of same-sign values -- the GPU result is accepted when it is within tol of the exact sum and
    no further from the CPU result than the CPU result is from the exact sum (plus tol);
  * exp is CUDA's expf against the CPU's expf: at most 2 ulp apart.
"""
from __future__ import annotations

import numpy as np

SUM_RTOL = 1e-5
EXP_ULP = 2

INT_DTYPES = [np.int32, np.uint32, np.int64, np.uint64, np.int16, np.uint16, np.int8, np.uint8]
ALL_DTYPES = [np.float32] + INT_DTYPES


def make_values(rng: np.random.Generator, n: int, dtype, kind: str = "normal", extremes: bool = True) -> np.ndarray:
    dtype = np.dtype(dtype)
    if dtype == np.float32:
        if kind == "normal":
            return rng.standard_normal(n).astype(np.float32)
        if kind == "uniform":
            return rng.uniform(-1, 1, n).astype(np.float32)
        if kind == "ties":  # multiples of 1/256 in [0, 1): many equal values
            return (np.floor(rng.uniform(0, 1, n) * 256) / 256).astype(np.float32)
        if kind == "special":
            v = rng.standard_normal(n).astype(np.float32)
            pick = rng.integers(0, 10, n)
            v[pick == 0] = np.nan
            v[pick == 1] = np.inf
            v[pick == 2] = -np.inf
            v[pick == 3] = 0.0
            v[pick == 4] = -0.0
            if extremes:  # +-FLT_MAX: fp32 partial sums overflow in an order-dependent way
                v[pick == 5] = np.finfo(np.float32).max
                v[pick == 6] = -np.finfo(np.float32).max
            return v
        raise ValueError(kind)
    info = np.iinfo(dtype)
    if kind == "small":
        lo, hi = max(info.min, -1000), min(info.max, 1000)
    else:  # full range: sums wrap
        lo, hi = info.min, info.max
    return rng.integers(lo, hi, n, dtype=dtype, endpoint=True)


def strided_view(base: np.ndarray, shape, strides, offset: int = 0) -> np.ndarray:
    """A view of the 1-D array `base` with element strides and an element offset."""
    it = base.itemsize
    return np.lib.stride_tricks.as_strided(base[offset:], shape=tuple(shape), strides=tuple(s * it for s in strides))


def to_device(base: np.ndarray):
    import torch

    return torch.from_numpy(np.ascontiguousarray(base)).cuda()


def device_view(dbase, shape, strides, offset: int = 0):
    import torch

    return torch.as_strided(dbase, tuple(shape), tuple(strides), offset)


def canonical_nans(a: np.ndarray) -> np.ndarray:
    a = np.array(a, order="C", copy=True)
    if a.dtype.kind == "f":
        a[np.isnan(a)] = np.nan
    return a


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = canonical_nans(a)
    b = canonical_nans(b)
    return a.shape == b.shape and a.dtype == b.dtype and a.tobytes() == b.tobytes()


def assert_bits_equal(gpu: np.ndarray, cpu: np.ndarray, what: str = "") -> None:
    assert gpu.shape == cpu.shape, f"{what}: shape {gpu.shape} != {cpu.shape}"
    assert gpu.dtype == cpu.dtype, f"{what}: dtype {gpu.dtype} != {cpu.dtype}"
    if not bits_equal(gpu, cpu):
        gpu, cpu = canonical_nans(gpu), canonical_nans(cpu)
        g = gpu.reshape(-1).view(np.uint8).reshape(gpu.size, -1) if gpu.size else gpu
        c = cpu.reshape(-1).view(np.uint8).reshape(cpu.size, -1) if cpu.size else cpu
        bad = np.nonzero(np.any(g != c, axis=1))[0]
        i = bad[0]
        raise AssertionError(f"{what}: {bad.size} of {gpu.size} elements differ; first at flat {i}: "
                             f"gpu={gpu.reshape(-1)[i]!r} cpu={cpu.reshape(-1)[i]!r}")


def assert_sum_close(gpu: np.ndarray, cpu: np.ndarray, abs_sum: np.ndarray, what: str = "",
                     exact: np.ndarray | None = None) -> None:
    assert gpu.shape == cpu.shape, f"{what}: shape {gpu.shape} != {cpu.shape}"
    g = gpu.astype(np.float64)
    c = cpu.astype(np.float64)
    tol = SUM_RTOL * np.asarray(abs_sum, dtype=np.float64).reshape(g.shape) + 1e-30
    both_nan = np.isnan(g) & np.isnan(c)
    same_inf = np.isinf(g) & (g == c)
    with np.errstate(invalid="ignore"):
        ok = (np.abs(g - c) <= tol) | both_nan | same_inf
        if exact is not None:
            e = np.asarray(exact, dtype=np.float64).reshape(g.shape)
            ok |= (np.abs(g - e) <= tol) & (np.abs(g - c) <= np.abs(c - e) + tol)
    if not ok.all():
        i = np.argwhere(~ok)[0]
        raise AssertionError(f"{what}: {np.count_nonzero(~ok)} outputs outside 1e-5*sum|x|; first {tuple(i)}: "
                             f"gpu={g[tuple(i)]} cpu={c[tuple(i)]} tol={tol[tuple(i)]}")


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units in the last place between float32 arrays (NaN vs NaN counts as 0)."""
    ai = a.astype(np.float32).view(np.int32).astype(np.int64)
    bi = b.astype(np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    d = np.atleast_1d(np.abs(ai - bi))
    d[np.atleast_1d(np.isnan(a) & np.isnan(b))] = 0
    return d
