"""Generates tests/golden/ fixtures from the reference's own CPU code.

The reference ships no tests or golden vectors for this path, so the fixtures are made here:
small seeded inputs evaluated by oracle/_ref/libmtx_ref.so -- the reference's hot-path CPU
loops and shape helpers compiled unchanged from its tree by oracle/build_ref.py.  The inputs,
the op descriptions and the reference's outputs are stored; tests/test_golden.py checks the
oracle restatement (and the product's host-side shape folding) against them without needing
the reference tree.

    python tests/golden/make_golden.py        # rewrites cases.json and golden.npz
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import oracle  # noqa: E402
from tests.helpers import make_values, strided_view  # noqa: E402

DTYPES = ["float32", "int32", "uint32", "int64", "uint64", "int16", "uint16", "int8", "uint8"]


def main() -> int:
    ref = oracle.reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libmtx_ref.so is missing: run `python oracle/build.py` with the reference tree")
    rng = np.random.default_rng(20261201)
    arrays: dict[str, np.ndarray] = {}
    cases: list[dict] = []

    def put(arr: np.ndarray) -> str:
        key = f"a{len(arrays)}"
        arrays[key] = np.array(arr, order="C", copy=True)  # keeps 0-d outputs 0-d
        return key

    # reductions: contiguous, permuted, sliced and expanded views; every op and dtype
    views = [
        ([5, 7], [7, 1], 0), ([3, 4, 5], [20, 5, 1], 0), ([4, 6], [1, 4], 0), ([3, 5, 4], [20, 1, 5], 1),
        ([6, 9], [10, 1], 2), ([2, 3, 4, 5], [60, 20, 5, 1], 0), ([4, 8], [0, 1], 0), ([2, 1, 3, 1, 8], [24, 24, 8, 8, 1], 0),
        ([300], [1], 0), ([3, 130], [131, 1], 1), ([1, 1], [1, 1], 0), ([4, 0], [1, 1], 0),
    ]
    for dt in DTYPES:
        for shape, strides, off in views:
            need = off + sum((e - 1) * s for e, s in zip(shape, strides)) + 1 if all(shape) else off + 1
            kind = "special" if dt == "float32" else "full"
            base = make_values(rng, max(need, 1), dt, kind)
            if dt == "float32" and rng.random() < 0.5:
                base = (np.floor(rng.random(max(need, 1)) * 8) / 8 - 0.5).astype(np.float32)  # ties
            x = strided_view(base, shape, strides, off)
            bkey = put(base)
            for axis in range(len(shape)):
                for keep in (False, True):
                    for op in ("sum", "max", "min", "argmax", "argmin"):
                        out = ref.reduce(op, x, axis, keep)
                        cases.append(dict(kind="reduce", op=op, dtype=dt, input=bkey, shape=shape, strides=strides,
                                          offset=off, axis=axis, keepdims=keep, output=put(out)))

    # broadcast binary ops
    pairs = [([3, 1, 4], [1, 5, 4]), ([4], [3, 4]), ([2, 1], [1, 3]), ([1], [2, 2]), ([3, 4], [3, 4]),
             ([2, 1, 3, 1], [4, 1, 5]), ([], [])]
    for dt in DTYPES:
        for sa, sb in pairs:
            a = make_values(rng, int(np.prod(sa)), dt, "special" if dt == "float32" else "full").reshape(sa)
            b = make_values(rng, int(np.prod(sb)), dt, "special" if dt == "float32" else "full").reshape(sb)
            for op in ("add", "sub", "mul", "div", "max", "min"):
                bb = b
                if op == "div" and dt != "float32":
                    bb = b.copy()
                    bb[bb == 0] = 1
                    if dt.startswith("int"):
                        bb[bb == -1] = 3
                out = ref.binary(op, a, bb)
                cases.append(dict(kind="binary", op=op, dtype=dt, a=put(a), b=put(bb), output=put(out)))

    # exp
    for shape, strides, off in views[:10]:
        need = off + sum((e - 1) * s for e, s in zip(shape, strides)) + 1
        base = (rng.standard_normal(need) * 20).astype(np.float32)
        x = strided_view(base, shape, strides, off)
        cases.append(dict(kind="exp", dtype="float32", input=put(base), shape=shape, strides=strides, offset=off,
                          output=put(ref.exp(x))))

    # shape folding metadata
    for trial in range(300):
        dims = int(rng.integers(1, 7))
        shape = [int(v) for v in rng.choice([1, 2, 3, 5, 65536, 3000000000], dims)]
        strides = [[int(v) for v in rng.integers(0, 1 << 32, dims, dtype=np.uint64)] if rng.random() < 0.3 else
                   oracle.row_major(shape) for _ in range(3)]
        cap = int(rng.choice([0x7FFFFFFF, 0xFFFFFFFF, 100]))
        axis = int(rng.integers(0, dims))
        keep = bool(rng.integers(0, 2))
        outer = bool(rng.integers(0, 2))
        rec = dict(kind="collapse", shape=shape, strides=strides, cap=cap, axis=axis, keep=keep, outer=outer)
        rec["collapse"] = [ref.collapse(shape, *strides[:n], cap=cap) for n in (1, 2, 3)]
        rec["collapse_reduce"] = [
            ref.collapse_reduce(shape, *strides[:n], axis=axis, keep=keep, cap=cap, **({"outer": outer} if n == 2 else {}))
            for n in (1, 2, 3)]
        cases.append(rec)

    # the widened rows: Float16 / BFloat16 / Bool reductions and broadcasts, astype over every dtype
    # pair, exp / sqrt, equal, the make_pointwise family and its collapse, mean / rms / norm
    from tests.test_oracle_pin_pointwise import ALL_CODES, STORAGE, values

    for code in (1, 10, 7):
        for shape, strides, off in views[:8]:
            need = off + sum((e - 1) * s for e, s in zip(shape, strides)) + 1
            base = values(rng, code, need, special=code != 7)
            x = strided_view(base, shape, strides, off)
            bkey = put(base)
            for axis in range(len(shape)):
                for op in ("sum", "max", "min", "argmax", "argmin"):
                    out = ref.reduce(op, x, axis, False, dtype_code=code)
                    cases.append(dict(kind="reduce_code", op=op, code=code, input=bkey, shape=shape, strides=strides,
                                      offset=off, axis=axis, output=put(out)))
        for sa, sb in pairs[:6]:
            a = values(rng, code, int(np.prod(sa)), special=code != 7).reshape(sa)
            b = values(rng, code, int(np.prod(sb)), special=code != 7).reshape(sb)
            for op in ("add", "sub", "mul", "div", "max", "min", "equal"):
                bb = np.ones_like(b) if (code == 7 and op == "div") else b
                out = ref.binary(op, a, bb, dtype_code=code)
                cases.append(dict(kind="binary_code", op=op, code=code, a=put(a), b=put(bb), output=put(out)))
    for src in ALL_CODES:
        for dst in ALL_CODES:
            x = values(rng, src, 24, dst_code=dst, special=dst not in (2, 3, 4, 5, 6, 8, 11, 12)).reshape(4, 6)
            for view, mc in ((x, True), (x.T, False), (x[:, ::2], True)):
                out = ref.astype(view, STORAGE[dst], make_contig=mc, src_code=src, dst_code=dst)
                cases.append(dict(kind="astype", src=src, dst=dst, input=put(x), view=["plain", "T", "step2"][
                    0 if view is x else (1 if mc is False else 2)], make_contig=mc, output=put(np.ascontiguousarray(out))))
    for op in ("exp", "sqrt"):
        for dt in (np.float32, np.float16):
            x = np.abs(rng.standard_normal(60) * 5).astype(dt).reshape(5, 12) if op == "sqrt" else \
                (rng.standard_normal(60) * 5).astype(dt).reshape(5, 12)
            cases.append(dict(kind="unary", op=op, input=put(x), output=put(ref.unary(op, x.T))))
    for code in ALL_CODES:
        for s0, s1, s2 in (([3, 1, 5], [4, 5], [3, 4, 1]), ([6], [1], [6]), ([2, 3, 4], [3, 1], [4])):
            a = values(rng, code, int(np.prod(s0)), special=True).reshape(s0)
            b = values(rng, code, int(np.prod(s1)), special=True).reshape(s1)
            c = rng.integers(0, 2, int(np.prod(s2))).astype(np.bool_).reshape(s2)
            for op, ins in (("greater", [a, b]), ("less", [a, b]), ("where", [c, a, b]), ("floor", [a]), ("full", [b])) + \
                    ((("logical_and", [a, b]),) if code == 7 else ()):
                out = ref.pointwise(op, ins, dtype_code=code)
                cases.append(dict(kind="pointwise", op=op, code=code, inputs=[put(i) for i in ins], output=put(out)))
    from tests.test_oracle_pin_pointwise import _collapse_case

    for trial in range(200):
        shape, rows = _collapse_case(rng)
        try:
            want = ref.pointwise_collapse(shape, rows)
        except ValueError:
            want = None
        cases.append(dict(kind="pointwise_collapse", shape=shape, rows=rows, collapse=want))
    for code in ALL_CODES:
        x = values(rng, code, 4 * 70, special=False).reshape(4, 70)
        for kind in ("mean", "rms", "norm"):
            for axis in (0, 1):
                out, oc = ref.stat(kind, x, axis, False, dtype_code=code)
                cases.append(dict(kind="stat", stat=kind, code=code, input=put(x), axis=axis, out_code=oc,
                                  output=put(out)))

    (HERE / "cases.json").write_text(json.dumps(cases, separators=(",", ":")))
    np.savez_compressed(HERE / "golden.npz", **arrays)
    print(f"{len(cases)} cases, {len(arrays)} arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
