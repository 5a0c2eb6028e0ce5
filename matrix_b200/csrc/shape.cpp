// Host-side shape folding: the reference's collapse_dims / collapse_dims_reduce
// (Mods/Utils.mm:114-435), broadcast_shapes (Matrix.mm:161-232) and promote_types
// (Matrix.mm:107-109 over matrix.h:166-180).
//
// The kernels receive exactly the collapsed metadata these produce, so they must agree with
// the reference bit for bit, including its uint32 (`size_m`) arithmetic: the product of two
// extents compared against SIZE_CAP is a 32-bit product.  One generic fold serves the 1-, 2-
// and 3-operand variants: `K` stride arrays travel together, an axis merges into the previous
// slot when every operand is contiguous across the boundary and the merged extent stays
// within the cap, axes of extent 1 are dropped, and the inner axis' strides win.
#include <algorithm>
#include <cstdint>

#include "mtxc.h"
#include "promote.h"

namespace {

using size_m = uint32_t;

// collapse_dims: the first axis always opens slot 0 (even with extent 1).
template <int K>
uint32_t fold_dims(const uint32_t* shape, const uint32_t* const (&in)[K], uint32_t dims, uint64_t cap,
                   uint32_t* out_shape, uint32_t* const (&out)[K]) {
    if (dims == 0) return 0;
    uint32_t slot = 0;
    out_shape[0] = shape[0];
    for (int k = 0; k < K; ++k) out[k][0] = in[k][0];
    for (uint32_t i = 1; i < dims; ++i) {
        const size_m ext = shape[i];
        if (ext == 1) continue;
        bool joins = (size_m)(out_shape[slot] * ext) <= cap;
        for (int k = 0; k < K && joins; ++k) joins = out[k][slot] == (size_m)(in[k][i] * ext);
        if (joins) {
            out_shape[slot] = out_shape[slot] * ext;
        } else {
            ++slot;
            out_shape[slot] = ext;
        }
        for (int k = 0; k < K; ++k) out[k][slot] = in[k][i];
    }
    return slot + 1;
}

// collapse_dims_reduce: the reduced axis is a hard boundary (kept as its own slot only with
// keep_dims); with `shift_out` operand 0 (the output) has one axis fewer than the input, so
// its strides past the reduced axis are read one position to the left.
template <int K>
uint32_t fold_dims_reduce(const uint32_t* shape, const uint32_t* const (&in)[K], uint32_t dims, int axis,
                          bool keep_dims, bool shift_out, uint64_t cap, uint32_t* out_shape,
                          uint32_t* const (&out)[K]) {
    if (dims == 0) return 0;
    int slot = -1;
    bool boundary = false;
    for (int i = 0; i < (int)dims; ++i) {
        if (i == axis) {
            if (keep_dims) {
                ++slot;
                out_shape[slot] = shape[i];
                for (int k = 0; k < K; ++k) out[k][slot] = in[k][i];
            }
            boundary = true;
            continue;
        }
        const size_m ext = shape[i];
        if (ext == 1) continue;
        auto stride_of = [&](int k) -> size_m {
            const int at = (k == 0 && shift_out && axis < i) ? i - 1 : i;
            return in[k][at];
        };
        bool joins = !boundary && slot >= 0 && (size_m)(out_shape[slot] * ext) <= cap;
        for (int k = 0; k < K && joins; ++k) joins = out[k][slot] == (size_m)(stride_of(k) * ext);
        if (joins) {
            out_shape[slot] = out_shape[slot] * ext;
        } else {
            ++slot;
            out_shape[slot] = ext;
            boundary = false;
        }
        for (int k = 0; k < K; ++k) out[k][slot] = stride_of(k);
    }
    return (uint32_t)(slot + 1);
}

}  // namespace

extern "C" {

uint32_t mtxc_collapse_dims1(const uint32_t* shape, const uint32_t* s0, uint32_t dims, uint64_t cap,
                             uint32_t* out_shape, uint32_t* o0) {
    const uint32_t* const in[1] = {s0};
    uint32_t* const out[1] = {o0};
    return fold_dims<1>(shape, in, dims, cap, out_shape, out);
}

uint32_t mtxc_collapse_dims2(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, uint32_t dims,
                             uint64_t cap, uint32_t* out_shape, uint32_t* o0, uint32_t* o1) {
    const uint32_t* const in[2] = {s0, s1};
    uint32_t* const out[2] = {o0, o1};
    return fold_dims<2>(shape, in, dims, cap, out_shape, out);
}

uint32_t mtxc_collapse_dims3(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, const uint32_t* s2,
                             uint32_t dims, uint64_t cap, uint32_t* out_shape, uint32_t* o0, uint32_t* o1,
                             uint32_t* o2) {
    const uint32_t* const in[3] = {s0, s1, s2};
    uint32_t* const out[3] = {o0, o1, o2};
    return fold_dims<3>(shape, in, dims, cap, out_shape, out);
}

uint32_t mtxc_collapse_dims_reduce1(const uint32_t* shape, const uint32_t* s_out, uint32_t dims, int axis,
                                    int keep_dims, uint64_t cap, uint32_t* out_shape, uint32_t* o0) {
    const uint32_t* const in[1] = {s_out};
    uint32_t* const out[1] = {o0};
    return fold_dims_reduce<1>(shape, in, dims, axis, keep_dims != 0, false, cap, out_shape, out);
}

uint32_t mtxc_collapse_dims_reduce2(const uint32_t* shape, const uint32_t* s_out, const uint32_t* s_in,
                                    uint32_t dims, int axis, int keep_dims, int outer_collapsed, uint64_t cap,
                                    uint32_t* out_shape, uint32_t* o0, uint32_t* o1) {
    const uint32_t* const in[2] = {s_out, s_in};
    uint32_t* const out[2] = {o0, o1};
    return fold_dims_reduce<2>(shape, in, dims, axis, keep_dims != 0, outer_collapsed != 0, cap, out_shape, out);
}

uint32_t mtxc_collapse_dims_reduce3(const uint32_t* shape, const uint32_t* s_out, const uint32_t* s_b,
                                    const uint32_t* s_c, uint32_t dims, int axis, int keep_dims, uint64_t cap,
                                    uint32_t* out_shape, uint32_t* o0, uint32_t* o1, uint32_t* o2) {
    const uint32_t* const in[3] = {s_out, s_b, s_c};
    uint32_t* const out[3] = {o0, o1, o2};
    return fold_dims_reduce<3>(shape, in, dims, axis, keep_dims != 0, false, cap, out_shape, out);
}

int mtxc_broadcast_shapes(const uint32_t* shape1, const uint32_t* strides1, int dim1, const uint32_t* shape2,
                          const uint32_t* strides2, int dim2, uint32_t* out_shape, uint32_t* out_strides,
                          uint32_t* a_shape, uint32_t* a_strides, uint32_t* b_shape, uint32_t* b_strides) {
    if (dim1 < 0 || dim2 < 0 || dim1 > MTXC_MAX_DIMS || dim2 > MTXC_MAX_DIMS) return MTXC_ERR_INVALID_ARGUMENT;
    const int rank = std::max(dim1, dim2);
    // Align both operands to the right; missing leading axes take the other operand's extent
    // and stride 0.
    for (int o = 0; o < rank; ++o) {
        const int i1 = o - (rank - dim1), i2 = o - (rank - dim2);
        const bool has1 = i1 >= 0, has2 = i2 >= 0;
        const uint32_t e1 = has1 ? shape1[i1] : 0, e2 = has2 ? shape2[i2] : 0;
        a_strides[o] = has1 ? strides1[i1] : 0;
        b_strides[o] = has2 ? strides2[i2] : 0;
        a_shape[o] = has1 ? e1 : e2;
        b_shape[o] = has2 ? e2 : e1;
        if (!has1) {
            out_shape[o] = e2;
        } else if (!has2) {
            out_shape[o] = e1;
        } else if (e1 == e2) {
            out_shape[o] = e1;
        } else if (e1 == 1) {
            out_shape[o] = e2;
            a_shape[o] = e2;
            a_strides[o] = 0;
        } else if (e2 == 1) {
            out_shape[o] = e1;
            b_shape[o] = e1;
            b_strides[o] = 0;
        } else {
            return MTXC_ERR_SHAPE;
        }
    }
    size_m acc = 1;
    for (int o = rank - 1; o >= 0; --o) {
        out_strides[o] = acc;
        acc *= out_shape[o];
    }
    return MTXC_OK;
}

int mtxc_promote_types(int a, int b) {
    return mtxc::promote_code(a, b);
}

// make_pointwise's collapse (Matrix.mm:13537-13555).  Walks the output axes outermost first, skips
// extent-1 axes, and folds an axis into the last kept one when the merged extent stays <= INT32_MAX
// and, for every input, the kept axis' stride equals this axis' stride times its extent (64-bit
// comparison, as in the reference).  The merged axis keeps the inner axis' strides.
uint32_t mtxc_pointwise_collapse(const uint32_t* out_shape, uint32_t out_dims, const uint32_t* in_strides,
                                 uint32_t n_inputs, uint32_t* out_cshape, uint32_t* out_strides) {
    if (out_dims > MTXC_MAX_DIMS || n_inputs > 3) return UINT32_MAX;
    if (out_dims && (!out_shape || (n_inputs && !in_strides))) return UINT32_MAX;
    if (!out_cshape || (n_inputs && !out_strides)) return UINT32_MAX;
    uint64_t count = 1;
    for (uint32_t d = 0; d < out_dims; ++d) {
        if (out_shape[d] && count > UINT32_MAX / out_shape[d]) return UINT32_MAX;  // overflow_error there
        count *= out_shape[d];
    }
    for (uint32_t i = 0; i < MTXC_MAX_DIMS; ++i) {
        out_cshape[i] = 0;
        for (uint32_t k = 0; k < n_inputs; ++k) out_strides[k * MTXC_MAX_DIMS + i] = 0;
    }
    uint32_t n = 0;
    if (count == 0) return 0;
    for (uint32_t d = 0; d < out_dims; ++d) {
        const uint32_t ext = out_shape[d];
        if (ext == 1) continue;
        bool merge = n > 0 && (uint64_t)out_cshape[n - 1] * ext <= INT32_MAX;
        for (uint32_t k = 0; k < n_inputs && merge; ++k)
            merge = (uint64_t)out_strides[k * MTXC_MAX_DIMS + n - 1] == (uint64_t)in_strides[k * out_dims + d] * ext;
        const uint32_t t = merge ? n - 1 : n++;
        out_cshape[t] = merge ? out_cshape[t] * ext : ext;
        for (uint32_t k = 0; k < n_inputs; ++k) out_strides[k * MTXC_MAX_DIMS + t] = in_strides[k * out_dims + d];
    }
    return n;
}

}  // extern "C"
