"""The fused softmax (mtxc_softmax_lastdim) against the oracle's evaluation of the reference trace
m = x.max(-1, true); e = exp(x - m); y = e / e.sum(-1, true), primitive by primitive on the CPU.

Element-wise the fused kernel performs the same operations as the trace; only the fp32 summation
order of the row sum differs.  Outputs must agree with the trace to a relative 1e-5.  The trace's own
sequential fp32 row sum can drift further than that from the exact sum on long rows (tens of
thousands of positive terms); there the fused result is accepted when it is within 1e-5 of the exact
(fp64) softmax and no further from the trace than the trace is from exact -- the rule the float-sum
tests use (tests/helpers.py)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def trace_cpu(port, x):
    m = port.reduce("max", x, -1, True)
    e = port.exp(port.binary("sub", x, m))
    return port.binary("div", e, port.reduce("sum", e, -1, True))


def check(gpu, port, x, what=""):
    import torch

    y_cpu = trace_cpu(port, x)
    y = gpu.softmax_lastdim(torch.from_numpy(x).cuda())
    gpu.sync()
    g = y.cpu().numpy()
    assert g.shape == y_cpu.shape
    both_nan = np.isnan(g) & np.isnan(y_cpu)
    with np.errstate(invalid="ignore", over="ignore"):
        ok = both_nan | (np.abs(g - y_cpu) <= 1e-5 * np.abs(y_cpu))
        if not ok.all():
            x64 = x.astype(np.float64)
            m = np.max(np.where(np.isnan(x64), -np.inf, x64), axis=-1, keepdims=True)
            m = np.maximum(m, -np.finfo(np.float32).max)
            e = np.exp(x64 - m)
            y64 = e / e.sum(-1, keepdims=True)
            tol = 1e-5 * np.abs(y64)
            ok |= (np.abs(g - y64) <= tol) & (np.abs(g - y_cpu) <= np.abs(y_cpu - y64) + 1e-5 * np.abs(y_cpu))
    assert ok.all(), f"{what}: {np.count_nonzero(~ok)} mismatches, first {np.argwhere(~ok)[0]}"


@pytest.mark.parametrize("cols", [4, 64, 1000, 1024, 2048, 4092, 8192, 12000, 16384, 32768, 40000, 65536])
def test_fused_softmax_matches_trace(gpu, port, cols):
    rng = np.random.default_rng(cols)
    rows = max(1, (1 << 22) // cols)
    x = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    check(gpu, port, x, f"[{rows},{cols}]")


def test_fused_softmax_special_rows(gpu, port):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((8, 4096)) * 2).astype(np.float32)
    x[0, 17] = np.nan                 # a NaN poisons its row, as in the trace
    x[1, :] = -np.inf                 # max stays -FLT_MAX, e = 0, y = 0/0
    x[2, :] = 0.0                     # uniform row
    x[3, ::2] = -0.0
    x[4, :100] = 80.0                 # large values: x - m keeps exp in range
    x[5, 7] = np.inf                  # inf - inf = NaN for that element
    x[6, :] = np.float32(-3.4e38)
    check(gpu, port, x, "special")


def test_fused_softmax_rejects_unsupported_rows(gpu):
    import torch

    from matrix_b200 import MtxcError

    with pytest.raises(MtxcError):
        gpu.softmax_lastdim(torch.zeros((4, 1001), device="cuda"))           # not a multiple of 4
    with pytest.raises(MtxcError):
        gpu.softmax_lastdim(torch.zeros((2, 65540), device="cuda"))          # longer than the max row


@pytest.mark.slow
def test_config5a_fused_full(gpu, port):
    """C5a at full size: f32 [8192, 32768] ~ N(0, 4)."""
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((8192, 32768), dtype=np.float32) * 2).astype(np.float32)
    check(gpu, port, x, "C5a")
