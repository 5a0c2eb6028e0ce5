"""Build recipe for oracle/_ref/libmtx_ref.so: the reference's OWN CPU code for the hot path.

TEST INFRASTRUCTURE ONLY (the checker, never the product).

The reference (AlanAditya/matrix) is Objective-C++ on Metal and cannot be built on Linux as a
whole.  Its hot-path CPU evaluation, however, is plain C++ sitting inside Objective-C++
methods: the scalar loops of the reduction and broadcast backends and the shape-folding
helpers.  This recipe reads those pieces from where they lie in the reference tree, verifies
each anchor, and compiles them unchanged, together with a small prelude (type aliases for the
ARM half types) and C-ABI wrappers written here, into ``oracle/_ref/libmtx_ref.so``.  The
generated source and the library stay in ``oracle/_ref/`` (git-ignored); nothing from the
reference is committed.

Pieces taken verbatim (file, anchor; the reference line numbers at the time of writing):
  Mods/Utils.h       size_m, MAX_TENSOR_DIMS, CollapsedDims{,_2,_3}          (125-149)
  Mods/Utils.mm      collapse_dims x3, collapse_dims_reduce x3               (114-202, 270-435)
  matrix.h           enum dtype (35-51), type_rules (166-180), SharedArrayDescriptor (184-205),
                     BroadcastDescriptor (223-236), array_descriptor (238-251),
                     dtype_lowest / dtype_max (271-282), dispatch_type (284-334),
                     dispatch_float_type (339-354)
  Matrix.mm          promote_types (107-109), descriptor helpers (131-159), broadcast_shapes
                     (161-232), CPU loops of sum (15188-15207), max (14895-14914), min
                     (15039-15058), argmax (16279-16302), argmin (16434-16457), broadcast
                     add/mul/sub/div lambdas (7475, 7546, 7614, 7683), max(a,b) (13459-13474),
                     min(a,b) (14764-14781), exp (7014-7063), the sqrt lambda (6878-6925),
                     the equal loop (14522-14538), make_pointwise's collapse (13544-13556), the
                     CPU backends greater / less / logical_and / where / floor / full
                     (13741-14166), arctan2 / arcsin (13608-13738) and arange (14167-14180)
  matrix.h           dtype_cast (260-267), copyCPUinplaceTypeCasted (1474-1544)
  primitives.cpp     ElementwiseDims (6614-6618)
The member functions are compiled as members of a small stand-in `matrix` struct and stand-in
primitive structs that carry only the fields those functions read.

Usage: ``python oracle/build_ref.py [--reference PATH]``.  The reference root defaults to the
``reference_path`` recorded in BASELINE.json at the repository root, or $MTX_REFERENCE_ROOT.
Exits 0 without building when the reference tree is absent (the GPU box only uses the
prebuilt library).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libmtx_ref.so"


def reference_root(cli: str | None) -> Path | None:
    if cli:
        return Path(cli)
    env = os.environ.get("MTX_REFERENCE_ROOT")
    if env:
        return Path(env)
    try:
        return Path(json.loads((REPO / "BASELINE.json").read_text())["reference_path"])
    except Exception:
        return None


class Source:
    def __init__(self, path: Path):
        self.path = path
        self.lines = path.read_text(errors="replace").splitlines()

    def find(self, pattern: str, after: int = 0, occurrence: int = 1) -> int:
        """0-based index of the `occurrence`-th line at or after `after` containing `pattern`."""
        seen = 0
        for i in range(after, len(self.lines)):
            if pattern in self.lines[i] and not self.lines[i].lstrip().startswith("//"):
                seen += 1
                if seen == occurrence:
                    return i
        raise SystemExit(f"build_ref: anchor not found in {self.path.name}: {pattern!r}")

    def block(self, start: int, statement: bool) -> tuple[int, int, str]:
        """Text from line `start` until its braces balance.

        statement=True also requires the terminating ';' (lambdas, `dispatch_type(...);`,
        struct/enum definitions).  Line comments are ignored when counting braces.
        """
        depth = 0
        opened = False
        out = []
        for i in range(start, len(self.lines)):
            line = self.lines[i]
            out.append(line)
            code = re.sub(r"//.*", "", line)
            code = re.sub(r'"(\\.|[^"\\])*"', '""', code)
            for ch in code:
                if ch == "{":
                    depth += 1
                    opened = True
                elif ch == "}":
                    depth -= 1
            if opened and depth == 0:
                if not statement or code.rstrip().endswith(";"):
                    return start, i, "\n".join(out)
        raise SystemExit(f"build_ref: unbalanced block at {self.path.name}:{start + 1}")

    def lines_between(self, start: int, end: int) -> str:
        return "\n".join(self.lines[start:end + 1])


PRELUDE = r"""
// Generated by oracle/build_ref.py from the reference tree.  Not committed.
#include <algorithm>
#include <atomic>
#include <cassert>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <new>
#include <stdexcept>
#include <type_traits>
#include <utility>
// The reference uses the ARM half types from <arm_fp16.h> / <arm_bf16.h>.
using float16_t = _Float16;
using bfloat16_t = __bf16;
struct complex64 { float re, im; };
// libstdc++ on x86 has no std::exp overload for _Float16 (the reference's fp16 exp evaluates in
// float and rounds back); give it one so the fp16 instantiation of the exp loop compiles.
namespace std { inline _Float16 exp(_Float16 x) { return (_Float16)::expf((float)x); } }
// Same for sqrt: evaluated in float (correctly rounded) and rounded once to half, which is what the
// reference's float16_t arithmetic does.
namespace std { inline _Float16 sqrt(_Float16 x) { return (_Float16)::sqrtf((float)x); } }
"""

WRAPPERS = r"""
// ---------------------------------------------------------------------------
// C-ABI wrappers (written by the recipe).  Each wrapper sets up exactly the locals the
// reference method has in scope at the fragment, then runs the fragment unchanged.
// ---------------------------------------------------------------------------
struct RefMat { void* buffer; size_t total_size; };

static void ref_sum_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 collapsed, uint32_t cdims,
                         size_m noOfOpp, size_m reduce_axis_stride) { @SUM@ }
static void ref_max_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 collapsed, uint32_t cdims,
                         size_m noOfOpp, size_m reduce_axis_stride) { @MAX@ }
static void ref_min_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 collapsed, uint32_t cdims,
                         size_m noOfOpp, size_m reduce_axis_stride) { @MIN@ }
static void ref_argmax_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 collapsed, uint32_t cdims,
                            size_m noOfOpp, size_m reduce_axis_stride) { @ARGMAX@ }
static void ref_argmin_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 collapsed, uint32_t cdims,
                            size_m noOfOpp, size_m reduce_axis_stride) { @ARGMIN@ }

static void ref_add_impl(dtype type, RefMat& result, void* buffer, RefMat& other, int cdims, size_m* strideA,
                         size_m* strideB, size_m* strideR) { @ADD@ dispatch_type(type, result.buffer, broadcasted_add); }
static void ref_mul_impl(dtype type, RefMat& result, void* buffer, RefMat& other, int cdims, size_m* strideA,
                         size_m* strideB, size_m* strideR) { @MUL@ dispatch_type(type, result.buffer, broadcasted_mul); }
static void ref_sub_impl(dtype type, RefMat& result, void* buffer, RefMat& other, int cdims, size_m* strideA,
                         size_m* strideB, size_m* strideR) { @SUB@ dispatch_type(type, result.buffer, broadcasted_sub); }
static void ref_div_impl(dtype type, RefMat& result, void* buffer, RefMat& other, int cdims, size_m* strideA,
                         size_m* strideB, size_m* strideR) { @DIV@ dispatch_type(type, result.buffer, broadcasted_div); }
static void ref_bmax_impl(dtype type, RefMat& result, void* buffer, RefMat& other, int cdims, size_m* strideA,
                          size_m* strideB, size_m* strideR) { @BMAX@ }
static void ref_bmin_impl(dtype type, RefMat& result, void* buffer, RefMat& other, int cdims, size_m* strideA,
                          size_m* strideB, size_m* strideR) { @BMIN@ }

static void ref_exp_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 res, uint32_t cdims,
                         size_t total_size) { @EXP@ }
static void ref_sqrt_impl(dtype type, RefMat& output, void* buffer, CollapsedDims_2 res, uint32_t cdims,
                          size_t total_size) { @SQRT@ dispatch_float_type(type, output.buffer, sqrt_cpu); }
// matrix::equal_backend's CPU branch, after its rank-0 rule (Matrix.mm:14480-14486)
static void ref_equal_impl(matrix& output, const matrix& a, const matrix& b, CollapsedDims_3 res) {
    if (res.out_dims == 0) {
        res.out_dims = 1;
        res.shape[0] = 1;
        res.stridesA[0] = res.stridesB[0] = res.stridesC[0] = 0;
    }
    uint32_t cdims = res.out_dims;
    if (output.total_size == 0) return;
    @EQUAL@
}

extern "C" {

int ref_reduce(int op, int dtype_code, void* out, const void* in, uint32_t rstride, uint32_t rlen,
               uint32_t cdims, const uint32_t* shape, const uint32_t* sA, const uint32_t* sB,
               uint64_t total_out) {
    CollapsedDims_2 c{};
    for (uint32_t i = 0; i < cdims && i < MAX_TENSOR_DIMS; ++i) {
        c.shape[i] = shape[i]; c.stridesA[i] = sA[i]; c.stridesB[i] = sB[i];
    }
    // the cdims == 0 rule the reference methods apply before their CPU branch
    if (cdims == 0) { cdims = 1; c.stridesA[0] = 1; c.stridesB[0] = 1; c.shape[0] = 1; }
    RefMat output{out, (size_t)total_out};
    try {
        switch (op) {
            case 0: ref_sum_impl((dtype)dtype_code, output, (void*)in, c, cdims, rlen, rstride); break;
            case 1: ref_max_impl((dtype)dtype_code, output, (void*)in, c, cdims, rlen, rstride); break;
            case 2: ref_min_impl((dtype)dtype_code, output, (void*)in, c, cdims, rlen, rstride); break;
            case 3: ref_argmax_impl((dtype)dtype_code, output, (void*)in, c, cdims, rlen, rstride); break;
            case 4: ref_argmin_impl((dtype)dtype_code, output, (void*)in, c, cdims, rlen, rstride); break;
            default: return -1;
        }
    } catch (...) { return -1; }
    return 0;
}

int ref_broadcast(int op, int dtype_code, void* out, const void* a, const void* b, uint32_t cdims,
                  const uint32_t* sR, const uint32_t* sA, const uint32_t* sB, uint64_t total) {
    size_m r[MAX_TENSOR_DIMS], x[MAX_TENSOR_DIMS], y[MAX_TENSOR_DIMS];
    for (uint32_t i = 0; i < cdims && i < MAX_TENSOR_DIMS; ++i) { r[i] = sR[i]; x[i] = sA[i]; y[i] = sB[i]; }
    RefMat result{out, (size_t)total};
    RefMat other{(void*)b, 0};
    dtype t = (dtype)dtype_code;
    try {
        switch (op) {
            case 0: ref_add_impl(t, result, (void*)a, other, (int)cdims, x, y, r); break;
            case 1: ref_sub_impl(t, result, (void*)a, other, (int)cdims, x, y, r); break;
            case 2: ref_mul_impl(t, result, (void*)a, other, (int)cdims, x, y, r); break;
            case 3: ref_div_impl(t, result, (void*)a, other, (int)cdims, x, y, r); break;
            case 4: ref_bmax_impl(t, result, (void*)a, other, (int)cdims, x, y, r); break;
            case 5: ref_bmin_impl(t, result, (void*)a, other, (int)cdims, x, y, r); break;
            default: return -1;
        }
    } catch (...) { return -1; }
    return 0;
}

int ref_exp(int dtype_code, void* out, const void* in, uint32_t cdims, const uint32_t* shape,
            const uint32_t* sOut, const uint32_t* sIn, uint64_t total) {
    CollapsedDims_2 res{};
    for (uint32_t i = 0; i < cdims && i < MAX_TENSOR_DIMS; ++i) {
        res.shape[i] = shape[i]; res.stridesA[i] = sOut[i]; res.stridesB[i] = sIn[i];
    }
    res.out_dims = cdims;
    RefMat output{out, (size_t)total};
    try { ref_exp_impl((dtype)dtype_code, output, (void*)in, res, cdims, (size_t)total); }
    catch (...) { return -1; }
    return 0;
}

static void copy_out(const size_m* src, uint32_t n, uint32_t* dst) { for (uint32_t i = 0; i < n; ++i) dst[i] = src[i]; }

uint32_t ref_collapse1(const uint32_t* shape, const uint32_t* s0, uint32_t dims, uint64_t cap,
                       uint32_t* oshape, uint32_t* os0) {
    CollapsedDims r = collapse_dims(shape, s0, dims, (size_t)cap);
    copy_out(r.shape, r.out_dims, oshape); copy_out(r.strides, r.out_dims, os0);
    return r.out_dims;
}
uint32_t ref_collapse2(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, uint32_t dims, uint64_t cap,
                       uint32_t* oshape, uint32_t* os0, uint32_t* os1) {
    CollapsedDims_2 r = collapse_dims(shape, s0, s1, dims, (size_t)cap);
    copy_out(r.shape, r.out_dims, oshape); copy_out(r.stridesA, r.out_dims, os0); copy_out(r.stridesB, r.out_dims, os1);
    return r.out_dims;
}
uint32_t ref_collapse3(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, const uint32_t* s2,
                       uint32_t dims, uint64_t cap, uint32_t* oshape, uint32_t* os0, uint32_t* os1, uint32_t* os2) {
    CollapsedDims_3 r = collapse_dims(shape, s0, s1, s2, dims, (size_t)cap);
    copy_out(r.shape, r.out_dims, oshape); copy_out(r.stridesA, r.out_dims, os0);
    copy_out(r.stridesB, r.out_dims, os1); copy_out(r.stridesC, r.out_dims, os2);
    return r.out_dims;
}
uint32_t ref_collapse_reduce1(const uint32_t* shape, const uint32_t* so, uint32_t dims, int axis, int keep,
                              uint64_t cap, uint32_t* oshape, uint32_t* oso) {
    CollapsedDims r = collapse_dims_reduce(shape, so, dims, axis, keep != 0, (size_t)cap);
    copy_out(r.shape, r.out_dims, oshape); copy_out(r.strides, r.out_dims, oso);
    return r.out_dims;
}
uint32_t ref_collapse_reduce2(const uint32_t* shape, const uint32_t* so, const uint32_t* si, uint32_t dims, int axis,
                              int keep, int outer, uint64_t cap, uint32_t* oshape, uint32_t* oso, uint32_t* osi) {
    CollapsedDims_2 r = collapse_dims_reduce(shape, so, si, dims, axis, keep != 0, outer != 0, (size_t)cap);
    copy_out(r.shape, r.out_dims, oshape); copy_out(r.stridesA, r.out_dims, oso); copy_out(r.stridesB, r.out_dims, osi);
    return r.out_dims;
}
uint32_t ref_collapse_reduce3(const uint32_t* shape, const uint32_t* so, const uint32_t* sb, const uint32_t* sc,
                              uint32_t dims, int axis, int keep, uint64_t cap, uint32_t* oshape, uint32_t* oso,
                              uint32_t* osb, uint32_t* osc) {
    CollapsedDims_3 r = collapse_dims_reduce(shape, so, sb, sc, dims, axis, keep != 0, (size_t)cap);
    copy_out(r.shape, r.out_dims, oshape); copy_out(r.stridesA, r.out_dims, oso);
    copy_out(r.stridesB, r.out_dims, osb); copy_out(r.stridesC, r.out_dims, osc);
    return r.out_dims;
}

static array_descriptor make_desc(const uint32_t* shape, const uint32_t* strides, int dims) {
    array_descriptor d;
    std::memset(&d, 0, sizeof(d));
    if (dims > SBO_MAX_DIMS) {
        d.shared_arr_desc = SharedArrayDescriptor::create(dims);
        for (int i = 0; i < dims; ++i) { d.shared_arr_desc->shape()[i] = shape[i]; d.shared_arr_desc->strides(dims)[i] = strides[i]; }
    } else {
        for (int i = 0; i < dims; ++i) { d.inline_buffer[i] = shape[i]; d.inline_buffer[SBO_MAX_DIMS + i] = strides[i]; }
    }
    return d;
}

int ref_broadcast_shapes(const uint32_t* shape1, const uint32_t* strides1, int dim1, const uint32_t* shape2,
                         const uint32_t* strides2, int dim2, uint32_t* out_shape, uint32_t* out_strides,
                         uint32_t* a_shape, uint32_t* a_strides, uint32_t* b_shape, uint32_t* b_strides) {
    int od = std::max(dim1, dim2);
    array_descriptor d1 = make_desc(shape1, strides1, dim1);
    array_descriptor d2 = make_desc(shape2, strides2, dim2);
    array_descriptor out;
    std::memset(&out, 0, sizeof(out));
    if (od > SBO_MAX_DIMS) out.shared_arr_desc = SharedArrayDescriptor::create(od);
    BroadcastDescriptor* na = BroadcastDescriptor::create(od);
    BroadcastDescriptor* nb = BroadcastDescriptor::create(od);
    int rc = 0;
    try {
        broadcast_shapes(d1, d2, out, na, nb, dim1, dim2);
        const size_m* os = od > SBO_MAX_DIMS ? out.shared_arr_desc->shape() : out.inline_buffer;
        const size_m* ot = od > SBO_MAX_DIMS ? out.shared_arr_desc->strides(od) : out.inline_buffer + SBO_MAX_DIMS;
        for (int i = 0; i < od; ++i) {
            out_shape[i] = os[i]; out_strides[i] = ot[i];
            a_shape[i] = na->shape()[i]; a_strides[i] = na->strides(od)[i];
            b_shape[i] = nb->shape()[i]; b_strides[i] = nb->strides(od)[i];
        }
    } catch (const std::invalid_argument&) { rc = -1; }
    d1.release(dim1); d2.release(dim2); out.release(od);
    BroadcastDescriptor::destroy(na); BroadcastDescriptor::destroy(nb);
    return rc;
}

int ref_promote(int a, int b) { return (int)promote_types((dtype)a, (dtype)b); }

int ref_unary(int op, int dtype_code, void* out, const void* in, uint32_t cdims, const uint32_t* shape,
              const uint32_t* sOut, const uint32_t* sIn, uint64_t total) {
    if (op == 0) return ref_exp(dtype_code, out, in, cdims, shape, sOut, sIn, total);
    CollapsedDims_2 res{};
    for (uint32_t i = 0; i < cdims && i < MAX_TENSOR_DIMS; ++i) {
        res.shape[i] = shape[i]; res.stridesA[i] = sOut[i]; res.stridesB[i] = sIn[i];
    }
    res.out_dims = cdims;
    RefMat output{out, (size_t)total};
    try { ref_sqrt_impl((dtype)dtype_code, output, (void*)in, res, cdims, (size_t)total); }
    catch (...) { return -1; }
    return 0;
}

int ref_astype(int dst_code, int src_code, void* out, const void* in, uint32_t dims, const uint32_t* shape,
               const uint32_t* sOut, const uint32_t* sIn, uint64_t total) {
    matrix o, i;
    o.type = (dtype)dst_code; o.buffer = out; o.total_size = (size_t)total; o.dims = dims;
    i.type = (dtype)src_code; i.buffer = (void*)in; i.total_size = (size_t)total; i.dims = dims;
    for (uint32_t k = 0; k < dims && k < MAX_TENSOR_DIMS; ++k) {
        o.shp[k] = i.shp[k] = shape[k]; o.str[k] = sOut[k]; i.str[k] = sIn[k];
    }
    try { matrix::copyCPUinplaceTypeCasted(o, i, 0); } catch (...) { return -1; }
    return 0;
}

uint32_t ref_pointwise_collapse(const uint32_t* out_shape, uint32_t out_dims, const uint32_t* in_strides,
                                uint32_t n, uint32_t* cshape, uint32_t* cstrides) {
    size_t count = 1;
    for (uint32_t d = 0; d < out_dims; ++d) {
        if (out_shape[d] && count > UINT32_MAX / out_shape[d]) return UINT32_MAX;
        count *= out_shape[d];
    }
    matrix out;
    out.dims = out_dims;
    for (uint32_t d = 0; d < out_dims; ++d) out.shp[d] = out_shape[d];
    PointwiseShim node;
    PointwiseShim* prim = &node;
    std::vector<int> inputs(n);
    size_m all_strides[3][MAX_TENSOR_DIMS]{};
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t d = 0; d < out_dims; ++d) all_strides[i][d] = in_strides[i * out_dims + d];
    @PWCOLLAPSE@
    const auto& cd = prim->collapsed_dims;
    for (uint32_t d = 0; d < MAX_TENSOR_DIMS; ++d) {
        cshape[d] = cd.shape[d];
        for (uint32_t i = 0; i < n; ++i) cstrides[i * MAX_TENSOR_DIMS + d] = cd.strides[i][d];
    }
    return cd.dims;
}

int ref_pointwise(int op, int dtype_code, void* out, const void* const* inputs, uint32_t n, uint32_t cdims,
                  const uint32_t* shape, const uint32_t* strides, uint64_t total) {
    static const uint32_t kArity[] = {2, 2, 2, 3, 1, 1, 2, 1};
    if (op < 0 || op > 7 || n != kArity[op]) return -1;
    ElementwiseDims cd{};
    cd.dims = cdims;
    for (uint32_t d = 0; d < cdims; ++d) {
        cd.shape[d] = shape[d];
        for (uint32_t i = 0; i < n; ++i) cd.strides[i][d] = strides[i * MAX_TENSOR_DIMS + d];
    }
    matrix in[3];
    for (uint32_t i = 0; i < n; ++i) { in[i].type = (dtype)dtype_code; in[i].buffer = (void*)inputs[i]; }
    matrix o;
    o.buffer = out;
    o.total_size = (size_t)total;
    try {
        switch (op) {
            case 0: { GreaterPrimitive p; p.a = in[0]; p.b = in[1]; p.collapsed_dims = cd; o.tape = &p; o.greater_backend_cpu(o); break; }
            case 1: { LessPrimitive p; p.a = in[0]; p.b = in[1]; p.collapsed_dims = cd; o.tape = &p; o.less_backend_cpu(o); break; }
            case 2: { LogicalAndPrimitive p; p.a = in[0]; p.b = in[1]; p.collapsed_dims = cd; o.tape = &p; o.logical_and_backend_cpu(o); break; }
            case 3: {
                WherePrimitive p; in[0].type = dtype::Bool;
                p.cond = in[0]; p.a = in[1]; p.b = in[2]; p.collapsed_dims = cd; o.tape = &p; o.where_backend_cpu(o); break;
            }
            case 4: { FloorPrimitive p; p.input = in[0]; p.collapsed_dims = cd; o.tape = &p; o.floor_backend_cpu(o); break; }
            case 6: { Arctan2Primitive p; p.a = in[0]; p.b = in[1]; p.collapsed_dims = cd; o.tape = &p; o.arctan2_backend_cpu(o); break; }
            case 7: { ArcsinPrimitive p; p.input = in[0]; p.collapsed_dims = cd; o.tape = &p; o.arcsin_backend_cpu(o); break; }
            default: { FullPrimitive p; p.value = in[0]; p.collapsed_dims = cd; o.tape = &p; o.full_backend_cpu(o); break; }
        }
    } catch (...) { return -1; }
    return 0;
}

int ref_arange(int dtype_code, void* out, const void* start, const void* step, uint64_t count) {
    matrix s, t, o;
    s.type = t.type = o.type = (dtype)dtype_code;
    s.buffer = (void*)start; t.buffer = (void*)step;
    o.buffer = out; o.total_size = (size_t)count;
    ArangePrimitive p; p.start = s; p.step = t; o.tape = &p;
    try { o.arange_backend_cpu(o); } catch (...) { return -1; }
    return 0;
}

int ref_equal(int dtype_code, void* out, const void* a_buf, const void* b_buf, uint32_t cdims, const uint32_t* shape,
              const uint32_t* sA, const uint32_t* sB, const uint32_t* sR, uint64_t total) {
    CollapsedDims_3 res{};
    res.out_dims = cdims;
    for (uint32_t i = 0; i < cdims && i < MAX_TENSOR_DIMS; ++i) {
        res.shape[i] = shape[i]; res.stridesA[i] = sA[i]; res.stridesB[i] = sB[i]; res.stridesC[i] = sR[i];
    }
    matrix a, b, output;
    a.buffer = (void*)a_buf; b.buffer = (void*)b_buf;
    output.type = (dtype)dtype_code; output.buffer = out; output.total_size = (size_t)total;
    try { ref_equal_impl(output, a, b, res); } catch (...) { return -1; }
    return 0;
}

}  // extern "C"
"""


def extract(ref: Path) -> tuple[str, dict]:
    utils_h = Source(ref / "Mods" / "Utils.h")
    utils_mm = Source(ref / "Mods" / "Utils.mm")
    matrix_h = Source(ref / "matrix.h")
    matrix_mm = Source(ref / "Matrix.mm")
    manifest: dict[str, list] = {}
    parts: list[str] = [PRELUDE]

    def take(src: Source, name: str, start: int, statement: bool) -> str:
        s, e, text = src.block(start, statement)
        manifest[name] = [src.path.name, s + 1, e + 1]
        return f"// ---- {src.path.name}:{s + 1}-{e + 1} ({name})\n{text}\n"

    # Mods/Utils.h: size_m .. CollapsedDims_3
    s = utils_h.find("using size_m = uint32_t;")
    e = utils_h.block(utils_h.find("struct CollapsedDims_3", s), True)[1]
    manifest["utils_h_types"] = ["Utils.h", s + 1, e + 1]
    parts.append(f"// ---- Utils.h:{s + 1}-{e + 1}\n" + utils_h.lines_between(s, e) + "\n")

    # matrix.h pieces
    parts.append(take(matrix_h, "dtype", matrix_h.find("enum class dtype"), True))
    parts.append("constexpr int kNumDtypes = 13;\n")
    parts.append(take(matrix_h, "type_rules", matrix_h.find("constexpr dtype type_rules[kNumDtypes][kNumDtypes]"), True))
    parts.append("dtype promote_types(dtype a, dtype b);\n")
    parts.append(take(matrix_h, "SharedArrayDescriptor", matrix_h.find("struct SharedArrayDescriptor {"), True))
    parts.append(take(matrix_h, "BroadcastDescriptor", matrix_h.find("struct alignas(size_m) BroadcastDescriptor"), True))
    sbo = matrix_h.find("static constexpr int SBO_MAX_DIMS")
    parts.append(f"// ---- matrix.h:{sbo + 1}\n{matrix_h.lines[sbo]}\n")
    parts.append(take(matrix_h, "array_descriptor", matrix_h.find("union array_descriptor"), True))
    for name, pat in (("dtype_lowest", "inline T dtype_lowest()"), ("dtype_max", "inline T dtype_max()")):
        i = matrix_h.find(pat)
        parts.append(f"// ---- matrix.h:{i}\n{matrix_h.lines[i - 1]}\n" + take(matrix_h, name, i, False))
    for name, pat in (("dispatch_type", "inline void dispatch_type(dtype type, void *buffer, Func &&function_to_run)"),
                      ("dispatch_float_type", "inline void dispatch_float_type(dtype type, void *buffer, Func &&function_to_run)")):
        i = matrix_h.find(pat)
        parts.append(f"{matrix_h.lines[i - 1]}\n" + take(matrix_h, name, i, False))

    # Matrix.mm: promote_types, descriptor helpers, broadcast_shapes
    parts.append(take(matrix_mm, "promote_types", matrix_mm.find("dtype promote_types(dtype a, dtype b) {"), False))
    parts.append(take(matrix_mm, "SharedArrayDescriptor::release", matrix_mm.find("void SharedArrayDescriptor::release() {"), False))
    parts.append(take(matrix_mm, "BroadcastDescriptor::shape", matrix_mm.find("inline size_m *BroadcastDescriptor::shape() {"), False))
    parts.append(take(matrix_mm, "BroadcastDescriptor::strides", matrix_mm.find("inline size_m *BroadcastDescriptor::strides(int dims) {"), False))
    parts.append(take(matrix_mm, "ensure_exclusive_out_desc", matrix_mm.find("static void ensure_exclusive_out_desc("), False))
    parts.append(take(matrix_mm, "broadcast_shapes", matrix_mm.find("void broadcast_shapes(const array_descriptor &arr_desc1,"), False))

    # Mods/Utils.mm: shape folding
    for name, pat in (
        ("collapse_dims_1", "CollapsedDims collapse_dims(const size_m shape[], const size_m strides[], const uint32_t dims"),
        ("collapse_dims_2", "CollapsedDims_2 collapse_dims(const size_m shape[], const size_m stridesA[], const size_m stridesB[], const uint32_t dims"),
        ("collapse_dims_3", "CollapsedDims_3 collapse_dims(const size_m shape[], const size_m stridesA[], const size_m stridesB[], const size_m stridesC[]"),
        ("collapse_dims_reduce_1", "CollapsedDims collapse_dims_reduce(const size_m shape[], const size_m stridesO[], const uint32_t dims"),
        ("collapse_dims_reduce_2", "CollapsedDims_2 collapse_dims_reduce(const size_m shape[], const size_m stridesO[], const size_m stridesI[]"),
        ("collapse_dims_reduce_3", "CollapsedDims_3 collapse_dims_reduce(const size_m shape[], const size_m stridesO[], const size_m stridesB[]"),
    ):
        parts.append(take(utils_mm, name, utils_mm.find(pat), False))

    # Matrix.mm: CPU loop fragments
    frags: dict[str, str] = {}

    def frag(key: str, method: str, pattern: str, occurrence: int = 1) -> None:
        m = matrix_mm.find(method)
        i = matrix_mm.find(pattern, after=m, occurrence=occurrence)
        s2, e2, text = matrix_mm.block(i, True)
        manifest[key] = ["Matrix.mm", s2 + 1, e2 + 1]
        frags[key] = f"\n// ---- Matrix.mm:{s2 + 1}-{e2 + 1} ({key})\n{text}\n"

    frag("SUM", "void matrix::sum(matrix& output, int axis, bool keepdims, ExecutionDevice exec_device)",
         "dispatch_type(type, output.buffer, [&](auto *out_data) {")
    frag("MAX", "void matrix::max(matrix& output, int axis, bool keepdims, ExecutionDevice exec_device)",
         "dispatch_type(type, output.buffer, [&](auto *out_data) {")
    frag("MIN", "void matrix::min(matrix& output, int axis, bool keepdims, ExecutionDevice exec_device)",
         "dispatch_type(type, output.buffer, [&](auto *out_data) {")
    frag("ARGMAX", "void matrix::argmax(matrix& output, int axis, bool keepdims, ExecutionDevice exec_device) const",
         "dispatch_type(type, buffer, [&](auto *in_data) {")
    frag("ARGMIN", "void matrix::argmin(matrix& output, int axis, bool keepdims, ExecutionDevice exec_device) const",
         "dispatch_type(type, buffer, [&](auto *in_data) {")
    frag("ADD", "void matrix::add_cpu_brodcasted(", "auto broadcasted_add = [&](auto *out_data) {")
    frag("MUL", "void matrix::multiply_cpu_brodcasted(", "auto broadcasted_mul = [&](auto *out_data) {")
    frag("SUB", "void matrix::subtract_cpu_brodcasted(", "auto broadcasted_sub = [&](auto *out_data) {")
    frag("DIV", "void matrix::divide_cpu_brodcasted(", "auto broadcasted_div = [&](auto *out_data) {")
    # max(a, b) / min(a, b): the second dispatch is the general (rank >= 1) loop
    frag("BMAX", "void matrix::max(const matrix& other, matrix& result, ExecutionDevice exec_device) const",
         "dispatch_type(type, result.buffer, [&](auto *out_data) {", occurrence=2)
    frag("BMIN", "void matrix::min(const matrix& other, matrix& result, ExecutionDevice exec_device) const",
         "dispatch_type(type, result.buffer, [&](auto *out_data) {", occurrence=2)
    frag("EXP", "void matrix::exp(matrix& output, ExecutionDevice exec_device)",
         "dispatch_float_type(type, output.buffer, [&](auto *out_data) {")

    frag("SQRT", "void matrix::sqrt(matrix& output, ExecutionDevice exec_device)",
         "auto sqrt_cpu = [&](auto *out_data) {")
    frag("EQUAL", "void matrix::equal_backend(matrix& output, ExecutionDevice exec_device)",
         "dispatch_type(output.type, output.buffer, [&](auto *out_data) {")
    # make_pointwise's collapse: the `if (count) { ... }` block
    mp = matrix_mm.find("matrix make_pointwise(const std::vector<matrix>& inputs,")
    i = matrix_mm.find("if (count) {", after=mp)
    s2, e2, text = matrix_mm.block(i, False)
    manifest["PWCOLLAPSE"] = ["Matrix.mm", s2 + 1, e2 + 1]
    frags["PWCOLLAPSE"] = f"\n// ---- Matrix.mm:{s2 + 1}-{e2 + 1} (make_pointwise collapse)\n{text}\n"

    # dtype_cast (matrix.h) and ElementwiseDims (primitives.cpp)
    i = matrix_h.find("inline Dst dtype_cast(Src v) {")
    parts.append(f"{matrix_h.lines[i - 1]}\n" + take(matrix_h, "dtype_cast", i, False))
    prim_cpp = Source(ref / "primitives.cpp")
    parts.append(take(prim_cpp, "ElementwiseDims", prim_cpp.find("struct ElementwiseDims {"), True))

    # stand-in matrix: the fields and no-op hooks the taken member functions use, with
    # copyCPUinplaceTypeCasted (an inline member in matrix.h) pasted into the struct body
    copy_cast = take(matrix_h, "copyCPUinplaceTypeCasted",
                     matrix_h.find("static void copyCPUinplaceTypeCasted(matrix &outMat, const matrix &inMat,"), False)
    # GCC 13 at -O3 miscompiles the vectorised Float16 <-> BFloat16 conversion loop (it stores the
    # source bits unconverted); the loop vectoriser is kept off for the stand-in matrix's members.
    parts.append(
        "#include <vector>\n"
        "#pragma GCC push_options\n"
        "#pragma GCC optimize(\"no-tree-loop-vectorize\")\n"
        "struct matrix {\n"
        "    dtype type = dtype::Float; void* buffer = nullptr; size_t total_size = 0; void* tape = nullptr;\n"
        "    uint32_t dims = 0; size_m shp[MAX_TENSOR_DIMS]{}; size_m str[MAX_TENSOR_DIMS]{};\n"
        "    const size_m* shape() const { return shp; }\n"
        "    const size_m* strides() const { return str; }\n"
        "    void update_from_trace() {}\n"
        "    void eval_cpu() {}\n"
        + copy_cast +
        "    void greater_backend_cpu(matrix& output); void less_backend_cpu(matrix& output);\n"
        "    void logical_and_backend_cpu(matrix& output); void where_backend_cpu(matrix& output);\n"
        "    void floor_backend_cpu(matrix& output); void full_backend_cpu(matrix& output);\n"
        "    void arctan2_backend_cpu(matrix& output); void arcsin_backend_cpu(matrix& output);\n"
        "    void arange_backend_cpu(matrix& output);\n"
        "};\n"
        "#pragma GCC pop_options\n"
        "struct GreaterPrimitive { matrix a, b; ElementwiseDims collapsed_dims; };\n"
        "struct LessPrimitive { matrix a, b; ElementwiseDims collapsed_dims; };\n"
        "struct LogicalAndPrimitive { matrix a, b; ElementwiseDims collapsed_dims; };\n"
        "struct WherePrimitive { matrix cond, a, b; ElementwiseDims collapsed_dims; };\n"
        "struct FloorPrimitive { matrix input; ElementwiseDims collapsed_dims; };\n"
        "struct FullPrimitive { matrix value; ElementwiseDims collapsed_dims; };\n"
        "struct Arctan2Primitive { matrix a, b; ElementwiseDims collapsed_dims; };\n"
        "struct ArcsinPrimitive { matrix input; ElementwiseDims collapsed_dims; };\n"
        "struct ArangePrimitive { matrix start, step; };\n"
        "struct PointwiseShim { ElementwiseDims collapsed_dims; };\n")
    for key, pat in (("greater_backend_cpu", "void matrix::greater_backend_cpu(matrix& output) {"),
                     ("less_backend_cpu", "void matrix::less_backend_cpu(matrix& output) {"),
                     ("logical_and_backend_cpu", "void matrix::logical_and_backend_cpu(matrix& output) {"),
                     ("where_backend_cpu", "void matrix::where_backend_cpu(matrix& output) {"),
                     ("floor_backend_cpu", "void matrix::floor_backend_cpu(matrix& output) {"),
                     ("full_backend_cpu", "void matrix::full_backend_cpu(matrix& output) {"),
                     ("arctan2_backend_cpu", "void matrix::arctan2_backend_cpu(matrix& output) {"),
                     ("arcsin_backend_cpu", "void matrix::arcsin_backend_cpu(matrix& output) {"),
                     ("arange_backend_cpu", "void matrix::arange_backend_cpu(matrix& output) {")):
        parts.append(take(matrix_mm, key, matrix_mm.find(pat), False))

    wrappers = WRAPPERS
    for key, text in frags.items():
        wrappers = wrappers.replace(f"@{key}@", text)
    parts.append(wrappers)
    return "\n".join(parts), manifest


def build(ref: Path | None = None, quiet: bool = False) -> bool:
    if ref is None or not (ref / "Matrix.mm").exists():
        if not quiet:
            print("build_ref: reference tree not present; skipping", file=sys.stderr)
        return False
    OUT_DIR.mkdir(exist_ok=True)
    src, manifest = extract(ref)
    cpp = OUT_DIR / "ref_hot_path.cpp"
    cpp.write_text(src)
    (OUT_DIR / "manifest.json").write_text(json.dumps(manifest, indent=1))
    cmd = ["g++", "-std=c++17", "-O3", "-ffp-contract=off", "-fPIC", "-shared", "-w",
           "-o", str(LIB), str(cpp)]
    subprocess.run(cmd, check=True)
    if not quiet:
        print(f"build_ref: built {LIB}")
    return True


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    args = ap.parse_args()
    build(reference_root(args.reference))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
