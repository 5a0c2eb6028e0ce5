"""The oracle (and the product's host-side shape folding) against the golden fixtures made from
the reference's own CPU code by tests/golden/make_golden.py.  Runs without the reference tree
and without a GPU."""
import json
from pathlib import Path

import numpy as np
import pytest

from tests.helpers import strided_view

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def golden():
    cases = json.loads((GOLDEN / "cases.json").read_text())
    arrays = np.load(GOLDEN / "golden.npz")
    return cases, {k: arrays[k] for k in arrays.files}


def test_fixture_inventory(golden):
    cases, _ = golden
    kinds = {c["kind"] for c in cases}
    assert kinds == {"reduce", "binary", "exp", "collapse"}
    assert {c["op"] for c in cases if c["kind"] == "reduce"} == {"sum", "max", "min", "argmax", "argmin"}
    assert {c["op"] for c in cases if c["kind"] == "binary"} == {"add", "sub", "mul", "div", "max", "min"}


def test_oracle_reductions_match_golden(golden, port):
    cases, arrays = golden
    n = 0
    for c in cases:
        if c["kind"] != "reduce":
            continue
        x = strided_view(arrays[c["input"]], c["shape"], c["strides"], c["offset"])
        got = port.reduce(c["op"], x, c["axis"], c["keepdims"])
        want = arrays[c["output"]]
        assert got.shape == want.shape and got.tobytes() == want.tobytes(), c
        n += 1
    assert n > 1000


def test_oracle_binary_ops_match_golden(golden, port):
    cases, arrays = golden
    for c in cases:
        if c["kind"] != "binary":
            continue
        got = port.binary(c["op"], arrays[c["a"]], arrays[c["b"]])
        want = arrays[c["output"]]
        assert got.shape == want.shape and got.tobytes() == want.tobytes(), c


def test_oracle_exp_matches_golden(golden, port):
    cases, arrays = golden
    for c in cases:
        if c["kind"] != "exp":
            continue
        x = strided_view(arrays[c["input"]], c["shape"], c["strides"], c["offset"])
        assert port.exp(x).tobytes() == arrays[c["output"]].tobytes(), c


def test_shape_folding_matches_golden(golden, port):
    from matrix_b200 import _abi

    L, arr = _abi.lib(), _abi.u32_array
    cases, _ = golden
    for c in cases:
        if c["kind"] != "collapse":
            continue
        shape, strides, cap = c["shape"], c["strides"], c["cap"]
        for n in (1, 2, 3):
            k, outs = c["collapse"][n - 1]
            assert list(port.collapse(shape, *strides[:n], cap=cap)) == [k, outs]
            o = [arr([]) for _ in range(n + 1)]
            kk = getattr(L, f"mtxc_collapse_dims{n}")(arr(shape), *[arr(s) for s in strides[:n]], len(shape), cap, *o)
            assert [kk, [list(v[:kk]) for v in o]] == [k, outs]
            k, outs = c["collapse_reduce"][n - 1]
            kw = dict(axis=c["axis"], keep=c["keep"], cap=cap)
            if n == 2:
                kw["outer"] = c["outer"]
            assert list(port.collapse_reduce(shape, *strides[:n], **kw)) == [k, outs]
            o = [arr([]) for _ in range(n + 1)]
            extra = [int(c["outer"])] if n == 2 else []
            kk = getattr(L, f"mtxc_collapse_dims_reduce{n}")(arr(shape), *[arr(s) for s in strides[:n]], len(shape),
                                                            c["axis"], int(c["keep"]), *extra, cap, *o)
            assert [kk, [list(v[:kk]) for v in o]] == [k, outs]
