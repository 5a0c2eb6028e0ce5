"""Config 5b at its full size against the oracle: the full Sum of 2^32 float32 values ~ N(0,1).

bench.py's headline evaluates x.sum(1).sum(0) on x = [8, 2^29] (2^32 elements exceed the reference's
32-bit size_m, so the tensor is held with two axes): mtxc_reduce for sum(1), then mtxc_reduce_sharded
with a one-rank communicator for sum(0) -- the path the bench times at N = 1.  The same seeded tensor
(bench.fill_c5b_rows) is copied to the host and summed by the oracle twice: as matrix::sum() means it,
one sequential fp32 sum over all 2^32 elements in memory order (Matrix.mm:15215-15218 over the Sum loop
15201-15204, with a 64-bit count), and as the composition x.sum(1).sum(0) of the reference's loop.  The
GPU result must satisfy the float-sum rule against each (within 1e-5 * sum|x| of the CPU, or of the
exact fp64 sum while no further from the CPU than the CPU is from exact).  16 GiB on the device and
16 GiB of host memory; about half a minute, most of it the oracle's sequential sum.
"""
import numpy as np
import pytest

from tests.helpers import assert_sum_close

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def test_c5b_full_sum_matches_oracle(gpu, port):
    import torch

    from bench import C5B_COLS, C5B_ROWS, fill_c5b_rows
    from matrix_b200.shard import NativeComm, reduce_sharded

    dev = torch.device("cuda", 0)
    x = torch.empty((C5B_ROWS, C5B_COLS), dtype=torch.float32, device=dev)
    fill_c5b_rows(x, 0)
    part = gpu.reduce("sum", x, 1)
    with NativeComm() as comm:
        got = reduce_sharded("sum", part, 0, C5B_ROWS, comm=comm)
        gpu.sync()
    got = np.float32(got.item())
    exact, absum = 0.0, 0.0
    host = np.empty(C5B_ROWS * C5B_COLS, dtype=np.float32)
    for r in range(C5B_ROWS):
        exact += float(x[r].sum(dtype=torch.float64).item())
        absum += float(x[r].abs().sum(dtype=torch.float64).item())
        torch.from_numpy(host[r * C5B_COLS:(r + 1) * C5B_COLS]).copy_(x[r])
    del x, part
    torch.cuda.empty_cache()

    flat = port.sum_flat(host)
    assert_sum_close(np.array([got]), np.array([flat]), np.array([absum]), "C5b vs the flat sequential sum",
                     exact=np.array([exact]))
    rows = port.reduce("sum", host.reshape(C5B_ROWS, C5B_COLS), 1)
    comp = port.reduce("sum", rows, 0)
    assert_sum_close(np.array([got]), np.array([comp]), np.array([absum]), "C5b vs sum(1).sum(0)",
                     exact=np.array([exact]))
    # the tolerance is not vacuous here: the GPU's tree sum is close to exact, far inside it
    assert abs(float(got) - exact) <= 1e-7 * absum
