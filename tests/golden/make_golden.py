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

    (HERE / "cases.json").write_text(json.dumps(cases, separators=(",", ":")))
    np.savez_compressed(HERE / "golden.npz", **arrays)
    print(f"{len(cases)} cases, {len(arrays)} arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
