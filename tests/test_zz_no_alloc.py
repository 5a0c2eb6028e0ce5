"""mtxc_reduce_noalloc: the reduction entry point for callers that cannot allocate device memory.

Some users of this library run where cudaMalloc is off limits -- inside another framework's memory
manager that owns all device memory, in latency-critical loops that cannot absorb the device-wide
synchronisation of cudaMalloc / cudaFree, or under a memory budget fixed up front.  mtxc_reduce keeps
its split-reduction partials in a workspace that mtxc_init allocates; mtxc_reduce_noalloc keeps them
in a fixed 4 MiB array that is part of the library's device image instead.  This file checks, through
the C ABI, that the allocation-free entry point returns what mtxc_reduce returns and what the CPU
oracle (the reference's CPU loops, restated) returns -- on two calls in a row, since every call reuses
the same array and finds the previous call's partials in it -- and that a reduction needing more scratch
than the array holds is refused with a clear error.  The refusal is reached through a test hook
(mtxc_debug_set_noalloc_limit, not part of the public header) that lowers the size the check compares
against: no reduction of a sensible size needs more than the 4 MiB array, which is the point of its size.

The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from tests.helpers import assert_bits_equal, assert_sum_close

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20

# (shape, reduced axis, dtype): each case splits its reduced axis across CTAs, so its partials
# live in the scratch array (checked below with mtxc_reduce_workspace_bytes)
CASES = [
    ([8, 1 << 22], 1, np.float32),       # few long rows: row kernel with split partials
    ([16, 4096, 256], 1, np.float32),    # strided axis, few outputs: column kernel with split partials
    ([3, 1 << 21], 1, np.int32),
    ([2, 8192, 128], 1, np.int64),
]
OPS = ["sum", "max", "min", "argmax", "argmin"]


def _lib():
    from matrix_b200 import _abi

    return _abi


def _call(entry, op, x, meta, out):
    abi = _lib()
    from matrix_b200 import backend

    shape, s_out, s_in = meta.arrays
    rc = getattr(abi.lib(), entry)(abi.REDUCE_OPS[op], backend.dtype_code(x.dtype), out.data_ptr(), x.data_ptr(),
                                   meta.rstride, meta.rlen, meta.cdims, shape, s_out, s_in)
    return rc


def _scratch_needed(op, x, meta):
    abi = _lib()
    from matrix_b200 import backend

    shape, s_out, s_in = meta.arrays
    need = ctypes.c_size_t()
    abi.check(abi.lib().mtxc_reduce_workspace_bytes(abi.REDUCE_OPS[op], backend.dtype_code(x.dtype), meta.rstride,
                                                    meta.rlen, meta.cdims, shape, s_out, s_in, ctypes.byref(need)))
    return need.value


def _inputs(shape, dtype, seed):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    if dtype == np.float32:
        # quantised values: many ties, so first-index tie-breaking is exercised
        return torch.floor(torch.randn(*shape, generator=g, device="cuda") * 64) / 64
    tdt = {np.int32: torch.int32, np.int64: torch.int64}[dtype]
    return torch.randint(-(1 << 30), 1 << 30, tuple(shape), generator=g, device="cuda", dtype=tdt)


def test_noalloc_matches_mtxc_reduce_on_consecutive_calls(gpu, port):
    import torch

    abi = _lib()
    for k, (shape, axis, dtype) in enumerate(CASES):
        x = _inputs(shape, dtype, 100 + k)
        xh = x.cpu().numpy()
        meta = gpu.reduce_meta(list(x.shape), list(x.stride()), axis)
        for op in OPS:
            need = _scratch_needed(op, x, meta)
            assert 0 < need <= SCRATCH_BYTES, f"{shape} {op}: expected split partials, need={need}"
            odt = torch.int32 if op.startswith("arg") else x.dtype
            want = torch.empty(meta.out_shape, dtype=odt, device="cuda")
            abi.check(_call("mtxc_reduce", op, x, meta, want))
            got = []
            for _ in range(2):  # two calls in a row through the same static scratch
                out = torch.full(meta.out_shape, 7, dtype=odt, device="cuda")
                abi.check(_call("mtxc_reduce_noalloc", op, x, meta, out))
                got.append(out)
            gpu.sync()
            w = want.cpu().numpy()
            cpu = port.reduce(op, xh, axis)
            for i, out in enumerate(got):
                g = out.cpu().numpy()
                tag = f"noalloc call {i + 1} {op} {shape} axis={axis} {np.dtype(dtype).name}"
                if op == "sum" and dtype == np.float32:
                    x64 = x.double()
                    abs_sum = x64.abs().sum(axis).cpu().numpy()
                    exact = x64.sum(axis).cpu().numpy()
                    assert_sum_close(g, w, abs_sum, tag + " vs mtxc_reduce", exact=exact)
                    assert_sum_close(g, cpu, abs_sum, tag + " vs the oracle", exact=exact)
                else:
                    assert_bits_equal(g, w, tag + " vs mtxc_reduce")
                    assert_bits_equal(g, cpu, tag + " vs the oracle")


def test_noalloc_refuses_reductions_beyond_its_scratch(gpu):
    import torch

    abi = _lib()
    L = abi.lib()
    L.mtxc_debug_set_noalloc_limit.restype = ctypes.c_size_t
    L.mtxc_debug_set_noalloc_limit.argtypes = [ctypes.c_size_t]
    x = _inputs([8, 1 << 22], np.float32, 7)
    meta = gpu.reduce_meta(list(x.shape), list(x.stride()), 1)
    need = _scratch_needed("sum", x, meta)
    limit = need // 2
    assert 0 < limit < SCRATCH_BYTES
    out = torch.full(meta.out_shape, 7.0, device="cuda")
    prev = L.mtxc_debug_set_noalloc_limit(limit)
    try:
        rc = _call("mtxc_reduce_noalloc", "sum", x, meta, out)
        assert rc == abi.ERR_WORKSPACE
        msg = L.mtxc_last_error().decode()
        assert "static scratch" in msg and str(limit) in msg and str(need) in msg, msg
        gpu.sync()
        assert bool((out == 7.0).all()), "a refused call must not write its output"
    finally:
        L.mtxc_debug_set_noalloc_limit(prev)
    # at the array's full size the same reduction runs, and the allocating entry point agrees
    abi.check(_call("mtxc_reduce_noalloc", "sum", x, meta, out))
    want = torch.empty_like(out)
    abi.check(_call("mtxc_reduce", "sum", x, meta, want))
    gpu.sync()
    assert torch.equal(out, want)
