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
    assert kinds == {"reduce", "binary", "exp", "collapse", "reduce_code", "binary_code", "astype", "unary",
                     "pointwise", "pointwise_collapse", "stat"}
    assert {(c["src"], c["dst"]) for c in cases if c["kind"] == "astype"} == {
        (s, d) for s in (0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12) for d in (0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12)}
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


def _same(got, want):
    got, want = np.asarray(got), np.asarray(want)
    return got.shape == want.shape and (got.tobytes() == want.tobytes() or np.array_equal(got, want, equal_nan=True))


def test_oracle_half_and_bool_match_golden(golden, port):
    cases, arrays = golden
    n = 0
    for c in cases:
        if c["kind"] == "reduce_code":
            x = strided_view(arrays[c["input"]], c["shape"], c["strides"], c["offset"])
            assert _same(port.reduce(c["op"], x, c["axis"], False, dtype_code=c["code"]), arrays[c["output"]]), c
            n += 1
        elif c["kind"] == "binary_code":
            got = port.binary(c["op"], arrays[c["a"]], arrays[c["b"]], dtype_code=c["code"])
            assert _same(got, arrays[c["output"]]), c
            n += 1
    assert n > 300


def test_oracle_astype_matches_golden(golden, port):
    from oracle.oracle import STORAGE

    cases, arrays = golden
    for c in cases:
        if c["kind"] != "astype":
            continue
        x = arrays[c["input"]]
        view = {"plain": x, "T": x.T, "step2": x[:, ::2]}[c["view"]]
        got = port.astype(view, STORAGE[c["dst"]], make_contig=c["make_contig"], src_code=c["src"], dst_code=c["dst"])
        assert _same(np.ascontiguousarray(got), arrays[c["output"]]), c


def test_oracle_unary_pointwise_stat_match_golden(golden, port):
    cases, arrays = golden
    seen = set()
    for c in cases:
        if c["kind"] == "unary":
            assert _same(port.unary(c["op"], arrays[c["input"]].T), arrays[c["output"]]), c
        elif c["kind"] == "pointwise":
            got = port.pointwise(c["op"], [arrays[k] for k in c["inputs"]], dtype_code=c["code"])
            assert _same(got, arrays[c["output"]]), c
        elif c["kind"] == "stat":
            got, oc = port.stat(c["stat"], arrays[c["input"]], c["axis"], False, dtype_code=c["code"])
            assert oc == c["out_code"] and _same(got, arrays[c["output"]]), c
        else:
            continue
        seen.add(c["kind"])
    assert seen == {"unary", "pointwise", "stat"}


def test_pointwise_collapse_matches_golden(golden, port):
    import ctypes as C

    from matrix_b200 import _abi

    L = _abi.lib()
    cases, _ = golden
    for c in cases:
        if c["kind"] != "pointwise_collapse":
            continue
        shape, rows, want = c["shape"], c["rows"], c["collapse"]
        if want is None:
            with pytest.raises(ValueError):
                port.pointwise_collapse(shape, rows)
            continue
        assert list(port.pointwise_collapse(shape, rows)) == want, c
        n, d = len(rows), len(shape)
        flat = (C.c_uint32 * max(1, n * d))(*[v for r in rows for v in r])
        cs, cst = _abi.u32_array([]), _abi.u32_array([], 3 * _abi.MAX_DIMS)
        k = L.mtxc_pointwise_collapse(_abi.u32_array(shape, max(d, 1)), d, flat, n, cs, cst)
        assert [k, list(cs[:k]), [list(cst[i * 8:i * 8 + k]) for i in range(n)]] == want, c
