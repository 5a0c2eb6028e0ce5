// Broadcasted binary ops (Add, Sub, Mul, Divide, Max, Min, Equal) for sm_100a.
//
// Replaces ComputeShaders/Brodcasted{Add,Sub,Mul,Divide,Max,Min}.metal behind
// add/subtract/multiply/divide_gpu_brodcasted (Matrix.mm:7709-8239), the METAL branch of
// matrix::max / min(other, result, dev) (Matrix.mm:13378-13476, 14683-14783) and Equal.metal behind
// matrix::equal_backend (Matrix.mm:14467-14539), which binds the same collapse_dims_3 metadata.
//
// Semantics follow the reference CPU loops (Matrix.mm:7475-7498 and siblings): result element
// gid, decoded axis by axis with the result strides, reads a and b through their own strides
// (0 on broadcast axes).  Float ops are one IEEE round-to-nearest operation each
// (__fadd_rn & co. keep the compiler from contracting anything), so results are bit-exact
// with the CPU; Max / Min keep `a` unless `b` is strictly greater / smaller (std::max /
// std::min); integer arithmetic wraps.
//
// Two kernels:
//   rows     the result is contiguous (row-major strides), and along the innermost axis each
//            operand is either contiguous or broadcast (stride 1 or 0) with 16-byte aligned
//            rows.  Rows of the innermost axis are spread over threads: a row is decoded once
//            (a few fast divisions) and then streamed with 128-bit loads of the contiguous
//            operands (through L2, where broadcast operands stay resident) and 128-bit
//            evict-first stores of the result.
//   generic  anything else: a grid-stride loop over elements with the reference's per-element
//            stride decode.
#include <algorithm>

#include "ops.cuh"

namespace mtxc {
namespace {

constexpr int kBlock = 256;
constexpr uint32_t kSegVecs = 4096;
// Rows per work unit of the grouped kernel.  Measured on B200 (C2, random data, 200 back-to-back
// launch pairs, one CTA per work unit): the row kernel 0.88 of the measured copy bandwidth, R = 2 0.89,
// R = 4 0.94, R = 8 0.96.
// Division is long per element (and 8 rows of its code use up to 255 registers): 2 rows for it.
template <int OP>
constexpr int kGroupRows = OP == MTXC_BINARY_DIV ? 2 : 8;

// ------------------------------------------------------------------------------------------
// rows: contiguous result, innermost operand strides in {0, 1}
// ------------------------------------------------------------------------------------------
struct RowArgs {
    void* r;
    const void* a;
    const void* b;
    uint32_t rows;       // number of innermost rows
    uint32_t vec_per_row;
    uint32_t seg_vecs;   // 16-byte vectors per work unit (a row is cut into segments of this size)
    uint32_t segs;       // segments per row
    uint32_t units;      // rows * segs (< 2^32)
    uint32_t tpr;        // threads per unit (power of two, <= kBlock)
    FastDiv seg_div;     // divides a unit index by segs
    Dims d;              // outer axes: shape (fast divisors), a strides in s0, b strides in s1
};

// A_VEC / B_VEC: the operand is contiguous along the row (read with 16-byte vectors) or broadcast
// along it (stride 0: one element per row, splatted).  Template flags keep the inner loop free of
// per-vector selects.
template <int OP, typename T, bool A_VEC, bool B_VEC>
__global__ void __launch_bounds__(kBlock) broadcast_rows_kernel(const RowArgs args) {
    constexpr int V = Vec16<T>::N;
    constexpr uint32_t U = 4;  // vectors in flight per thread
    const uint32_t rows_per_block = kBlock / args.tpr;
    const uint32_t sub = threadIdx.x / args.tpr;
    const uint32_t lane = threadIdx.x % args.tpr;
    const T* __restrict__ pa = static_cast<const T*>(args.a);
    const T* __restrict__ pb = static_cast<const T*>(args.b);
    T* __restrict__ pr = static_cast<T*>(args.r);
    const uint64_t row_len = (uint64_t)args.vec_per_row * V;
    const uint32_t units = args.units;

    for (uint32_t u = blockIdx.x * rows_per_block + sub; u < units; u += gridDim.x * rows_per_block) {
        uint32_t row = u, seg = 0;
        if (args.segs > 1) args.seg_div.divmod(u, row, seg);
        const uint32_t c_end = min(args.vec_per_row, (seg + 1) * args.seg_vecs);
        uint64_t oa = 0, ob = 0;
        uint32_t rem = row;
#pragma unroll 1
        for (int i = (int)args.d.n - 1; i >= 0; --i) {
            uint32_t q, idx;
            args.d.fdiv[i].divmod(rem, q, idx);
            oa += (uint64_t)idx * args.d.s0[i];
            ob += (uint64_t)idx * args.d.s1[i];
            rem = q;
        }
        const T* ra = pa + oa;
        const T* rb = pb + ob;
        T* rr = pr + (uint64_t)row * row_len;
        Vec16<T> sa, sb;
        if constexpr (!A_VEC) {
            const T v = ra[0];
#pragma unroll
            for (int j = 0; j < V; ++j) sa.v[j] = v;
        }
        if constexpr (!B_VEC) {
            const T v = rb[0];
#pragma unroll
            for (int j = 0; j < V; ++j) sb.v[j] = v;
        }
        uint32_t c = seg * args.seg_vecs + lane;
        for (; c + (U - 1) * args.tpr < c_end; c += U * args.tpr) {
            Vec16<T> xa[U], xb[U];
#pragma unroll
            for (uint32_t k = 0; k < U; ++k) {
                if constexpr (A_VEC) xa[k] = load_cached(ra + (uint64_t)(c + k * args.tpr) * V);
                else xa[k] = sa;
                if constexpr (B_VEC) xb[k] = load_cached(rb + (uint64_t)(c + k * args.tpr) * V);
                else xb[k] = sb;
            }
#pragma unroll
            for (uint32_t k = 0; k < U; ++k) {
                store_stream(rr + (uint64_t)(c + k * args.tpr) * V, apply_vec<OP, T>(xa[k], xb[k]));
            }
        }
        for (; c < c_end; c += args.tpr) {
            const Vec16<T> xa = A_VEC ? load_cached(ra + (uint64_t)c * V) : sa;
            const Vec16<T> xb = B_VEC ? load_cached(rb + (uint64_t)c * V) : sb;
            store_stream(rr + (uint64_t)c * V, apply_vec<OP, T>(xa, xb));
        }
    }
}

// ------------------------------------------------------------------------------------------
// grouped rows: both operands contiguous along the row, and one of them broadcast (stride 0) along
// the next axis out.  Consecutive rows of that axis then share that operand's row (C2: every
// a[i, 0, :] serves the 512 rows b[0, j, :]).  A work unit covers R such rows: the shared operand's
// vector is loaded once for R outputs, the other operand's R vectors once each, so the reads from L2
// per 16-byte output vector drop from 2 to (1 + R) / R.  The operands live in L2 (C2: 12 MiB); what
// the row kernel spends there is the SM <-> L2 traffic of two reads next to every write.
// ------------------------------------------------------------------------------------------
struct GroupArgs {
    void* r;
    const void* a;
    const void* b;
    uint32_t vec_per_row;
    uint32_t seg_vecs;
    uint32_t segs;
    uint32_t extent;      // rows along the grouped axis (shape[k-1])
    uint32_t groups;      // ceil(extent / R)
    uint32_t units;       // (rows / extent) * groups * segs
    uint32_t tpr;
    uint32_t other_stride;  // the non-shared operand's stride along the grouped axis
    FastDiv seg_div;
    FastDiv group_div;    // divides by groups
    Dims d;               // axes 0 .. k-1 (the grouped axis included): shape, a strides (s0), b strides (s1)
};

template <int OP, typename T, bool SHARE_A, int R>
__global__ void __launch_bounds__(kBlock) broadcast_group_kernel(const GroupArgs g) {
    constexpr int V = Vec16<T>::N;
    constexpr uint32_t U = 2;  // vector positions in flight per thread (each with 1 + R loads)
    const uint32_t rows_per_block = kBlock / g.tpr;
    const uint32_t sub = threadIdx.x / g.tpr;
    const uint32_t lane = threadIdx.x % g.tpr;
    const T* __restrict__ pa = static_cast<const T*>(g.a);
    const T* __restrict__ pb = static_cast<const T*>(g.b);
    T* __restrict__ pr = static_cast<T*>(g.r);
    const uint64_t row_len = (uint64_t)g.vec_per_row * V;
    for (uint32_t u = blockIdx.x * rows_per_block + sub; u < g.units; u += gridDim.x * rows_per_block) {
        uint32_t gu = u, seg = 0;
        if (g.segs > 1) g.seg_div.divmod(u, gu, seg);
        uint32_t outer, gi;
        g.group_div.divmod(gu, outer, gi);
        const uint32_t j0 = gi * R;
        const uint32_t nr = min((uint32_t)R, g.extent - j0);
        const uint32_t row0 = outer * g.extent + j0;
        uint64_t oa = 0, ob = 0;
        uint32_t rem = row0;
#pragma unroll 1
        for (int i = (int)g.d.n - 1; i >= 0; --i) {
            uint32_t q, idx;
            g.d.fdiv[i].divmod(rem, q, idx);
            oa += (uint64_t)idx * g.d.s0[i];
            ob += (uint64_t)idx * g.d.s1[i];
            rem = q;
        }
        const T* ps = SHARE_A ? pa + oa : pb + ob;  // shared along the group
        const T* po = SHARE_A ? pb + ob : pa + oa;  // one row per grouped index
        T* rr = pr + (uint64_t)row0 * row_len;
        const uint32_t c_end = min(g.vec_per_row, (seg + 1) * g.seg_vecs);
        uint32_t c = seg * g.seg_vecs + lane;
        if (nr == (uint32_t)R) {
            for (; c + (U - 1) * g.tpr < c_end; c += U * g.tpr) {
                Vec16<T> xs[U], xo[U][R];
#pragma unroll
                for (uint32_t k = 0; k < U; ++k) {
                    const uint64_t e = (uint64_t)(c + k * g.tpr) * V;
                    xs[k] = load_cached(ps + e);
#pragma unroll
                    for (int t = 0; t < R; ++t) xo[k][t] = load_cached(po + (uint64_t)t * g.other_stride + e);
                }
#pragma unroll
                for (uint32_t k = 0; k < U; ++k) {
                    const uint64_t e = (uint64_t)(c + k * g.tpr) * V;
#pragma unroll
                    for (int t = 0; t < R; ++t)
                        store_stream(rr + (uint64_t)t * row_len + e,
                                     SHARE_A ? apply_vec<OP, T>(xs[k], xo[k][t]) : apply_vec<OP, T>(xo[k][t], xs[k]));
                }
            }
        }
        // the tail of a segment, and every vector of a partial last group (extent not a multiple of R)
        for (; c < c_end; c += g.tpr) {
            const uint64_t e = (uint64_t)c * V;
            const Vec16<T> xs = load_cached(ps + e);
#pragma unroll 1
            for (uint32_t t = 0; t < nr; ++t) {
                const Vec16<T> xo = load_cached(po + (uint64_t)t * g.other_stride + e);
                store_stream(rr + (uint64_t)t * row_len + e,
                             SHARE_A ? apply_vec<OP, T>(xs, xo) : apply_vec<OP, T>(xo, xs));
            }
        }
    }
}

// ------------------------------------------------------------------------------------------
// generic: the reference's per-element decode (Matrix.mm:7486-7494)
// ------------------------------------------------------------------------------------------
struct GenericArgs {
    void* r;
    const void* a;
    const void* b;
    uint64_t total;
    uint32_t cdims;
    uint32_t sr[MTXC_MAX_DIMS];
    uint32_t sa[MTXC_MAX_DIMS];
    uint32_t sb[MTXC_MAX_DIMS];
    FastDiv fr[MTXC_MAX_DIMS];  // divisors = result strides (used when total < 2^32)
};

template <int OP, typename T, bool k32>
__global__ void __launch_bounds__(kBlock) broadcast_generic_kernel(const GenericArgs g) {
    const T* __restrict__ pa = static_cast<const T*>(g.a);
    const T* __restrict__ pb = static_cast<const T*>(g.b);
    T* __restrict__ pr = static_cast<T*>(g.r);
    for (uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < g.total;
         gid += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t ia = 0, ib = 0;
        if constexpr (k32) {
            uint32_t rem = (uint32_t)gid;
            for (uint32_t i = 0; i < g.cdims; ++i) {
                uint32_t q, r;
                g.fr[i].divmod(rem, q, r);
                ia += (uint64_t)q * g.sa[i];
                ib += (uint64_t)q * g.sb[i];
                rem = r;
            }
        } else {
            uint64_t rem = gid;
            for (uint32_t i = 0; i < g.cdims; ++i) {
                const uint64_t q = rem / g.sr[i];
                ia += q * g.sa[i];
                ib += q * g.sb[i];
                rem %= g.sr[i];
            }
        }
        pr[gid] = apply<OP, T>(pa[ia], pb[ib]);
    }
}

template <int OP, typename T>
__global__ void broadcast_scalar_kernel(void* r, const void* a, const void* b) {
    static_cast<T*>(r)[0] = apply<OP, T>(static_cast<const T*>(a)[0], static_cast<const T*>(b)[0]);
}

template <int OP, typename T>
int launch_broadcast(void* r, const void* a, const void* b, uint32_t cdims, const uint32_t* shape,
                     const uint32_t* sr, const uint32_t* sa, const uint32_t* sb, int sm_count, cudaStream_t stream) {
    constexpr uint32_t V = Vec16<T>::N;
    if (cdims == 0) {
        broadcast_scalar_kernel<OP, T><<<1, 1, 0, stream>>>(r, a, b);
        return check_launch("broadcast_scalar_kernel");
    }
    const uint64_t total = product(shape, cdims);
    if (total == 0) return MTXC_OK;
    const uint32_t k = cdims - 1;
    // An operand read with 16-byte vectors (inner stride 1) needs aligned row starts; one that
    // is broadcast along the row (inner stride 0) is read as a single element per row.
    bool rows_ok = is_row_major(shape, sr, cdims) && sr[k] == 1 && (sa[k] <= 1) && (sb[k] <= 1) &&
                   shape[k] % V == 0 && aligned16(r) && (sa[k] == 0 || aligned16(a)) &&
                   (sb[k] == 0 || aligned16(b)) && total / shape[k] < (1ull << 32);
    for (uint32_t i = 0; i < k && rows_ok; ++i)
        rows_ok = shape[i] == 1 || ((sa[k] == 0 || sa[i] % V == 0) && (sb[k] == 0 || sb[i] % V == 0));
    // grouped rows: both operands contiguous along the row, exactly one broadcast along axis k - 1
    if (rows_ok && k >= 1 && sa[k] == 1 && sb[k] == 1 && (sa[k - 1] == 0) != (sb[k - 1] == 0) &&
        shape[k - 1] >= (uint32_t)kGroupRows<OP>) {
        const bool share_a = sa[k - 1] == 0;
        GroupArgs g{};
        g.r = r;
        g.a = a;
        g.b = b;
        g.vec_per_row = shape[k] / V;
        g.seg_vecs = std::min<uint32_t>(g.vec_per_row, kSegVecs);
        g.segs = (g.vec_per_row + g.seg_vecs - 1) / g.seg_vecs;
        g.extent = shape[k - 1];
        g.groups = (g.extent + kGroupRows<OP> - 1) / kGroupRows<OP>;
        g.other_stride = share_a ? sb[k - 1] : sa[k - 1];
        const uint64_t units = (total / shape[k] / g.extent) * g.groups * g.segs;
        uint32_t tpr = 1;
        while (tpr < g.seg_vecs && tpr < (uint32_t)kBlock) tpr <<= 1;
        g.tpr = tpr;
        g.seg_div = FastDiv(g.segs);
        g.group_div = FastDiv(g.groups);
        g.d.n = k;
        for (uint32_t i = 0; i < k; ++i) {
            g.d.shape[i] = shape[i];
            g.d.s0[i] = sa[i];
            g.d.s1[i] = sb[i];
            g.d.fdiv[i] = FastDiv(shape[i]);
        }
        if (units < (1ull << 31)) {
            g.units = (uint32_t)units;
            // one CTA per work unit (against 3 and 8 CTAs per SM looping over the units: 0.91 -> 0.94 at R = 4)
            const uint32_t rows_per_block = kBlock / tpr;
            const uint64_t blocks = (units + rows_per_block - 1) / rows_per_block;
            if (share_a) broadcast_group_kernel<OP, T, true, kGroupRows<OP>><<<(unsigned)blocks, kBlock, 0, stream>>>(g);
            else broadcast_group_kernel<OP, T, false, kGroupRows<OP>><<<(unsigned)blocks, kBlock, 0, stream>>>(g);
            return check_launch("broadcast_group_kernel");
        }
    }
    if (rows_ok) {
        RowArgs args{};
        args.r = r;
        args.a = a;
        args.b = b;
        args.rows = (uint32_t)(total / shape[k]);
        args.vec_per_row = shape[k] / V;
        // long rows are cut into segments of kSegVecs vectors so the grid has work for every SM
        args.seg_vecs = std::min<uint32_t>(args.vec_per_row, kSegVecs);
        args.segs = (args.vec_per_row + args.seg_vecs - 1) / args.seg_vecs;
        uint32_t tpr = 1;
        while (tpr < args.seg_vecs && tpr < (uint32_t)kBlock) tpr <<= 1;
        args.tpr = tpr;
        args.seg_div = FastDiv(args.segs);
        args.d.n = k;
        for (uint32_t i = 0; i < k; ++i) {
            args.d.shape[i] = shape[i];
            args.d.s0[i] = sa[i];
            args.d.s1[i] = sb[i];
            args.d.fdiv[i] = FastDiv(shape[i]);
        }
        const uint32_t rows_per_block = kBlock / tpr;
        const uint64_t units = (uint64_t)args.rows * args.segs;
        args.units = (uint32_t)units;
        uint64_t blocks = (units + rows_per_block - 1) / rows_per_block;
        // 3 CTAs (24 warps) per SM: measured on B200 with random data (where the stream runs into the
        // 1 kW power cap) against 2, 4 and 6 per SM, this grid is fastest both in short bursts
        // (~6.3 TB/s) and sustained over a thousand launches (~5.5 TB/s)
        blocks = std::min<uint64_t>(blocks, (uint64_t)sm_count * 3);
        if (sa[k] && sb[k]) broadcast_rows_kernel<OP, T, true, true><<<(unsigned)blocks, kBlock, 0, stream>>>(args);
        else if (sa[k]) broadcast_rows_kernel<OP, T, true, false><<<(unsigned)blocks, kBlock, 0, stream>>>(args);
        else if (sb[k]) broadcast_rows_kernel<OP, T, false, true><<<(unsigned)blocks, kBlock, 0, stream>>>(args);
        else broadcast_rows_kernel<OP, T, false, false><<<(unsigned)blocks, kBlock, 0, stream>>>(args);
        return check_launch("broadcast_rows_kernel");
    }
    GenericArgs g{};
    g.r = r;
    g.a = a;
    g.b = b;
    g.total = total;
    g.cdims = cdims;
    for (uint32_t i = 0; i < cdims; ++i) {
        if (sr[i] == 0) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary: zero result stride");
        g.sr[i] = sr[i];
        g.sa[i] = sa[i];
        g.sb[i] = sb[i];
        g.fr[i] = FastDiv(sr[i]);
    }
    const uint64_t blocks = std::min<uint64_t>((total + kBlock - 1) / kBlock, (uint64_t)sm_count * 16);
    if (total < (1ull << 32)) broadcast_generic_kernel<OP, T, true><<<(unsigned)blocks, kBlock, 0, stream>>>(g);
    else broadcast_generic_kernel<OP, T, false><<<(unsigned)blocks, kBlock, 0, stream>>>(g);
    return check_launch("broadcast_generic_kernel");
}

template <typename T>
int launch_broadcast_op(int op, void* r, const void* a, const void* b, uint32_t cdims, const uint32_t* shape,
                        const uint32_t* sr, const uint32_t* sa, const uint32_t* sb, int sms, cudaStream_t st) {
    switch (op) {
        case MTXC_BINARY_ADD: return launch_broadcast<MTXC_BINARY_ADD, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        case MTXC_BINARY_SUB: return launch_broadcast<MTXC_BINARY_SUB, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        case MTXC_BINARY_MUL: return launch_broadcast<MTXC_BINARY_MUL, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        case MTXC_BINARY_DIV: return launch_broadcast<MTXC_BINARY_DIV, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        case MTXC_BINARY_MAX: return launch_broadcast<MTXC_BINARY_MAX, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        case MTXC_BINARY_MIN: return launch_broadcast<MTXC_BINARY_MIN, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        case MTXC_BINARY_EQUAL: return launch_broadcast<MTXC_BINARY_EQUAL, T>(r, a, b, cdims, shape, sr, sa, sb, sms, st);
        default: return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary: unknown op");
    }
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_broadcast_binary(int op, int dtype, void* r, const void* a, const void* b, uint32_t cdims,
                                     const uint32_t* shape, const uint32_t* r_strides, const uint32_t* a_strides,
                                     const uint32_t* b_strides) {
    if (int rc = require_init()) return rc;
    if (op < MTXC_BINARY_ADD || op > MTXC_BINARY_EQUAL)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary: unknown op");
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary: cdims > MTXC_MAX_DIMS");
    if (cdims && (!shape || !r_strides || !a_strides || !b_strides))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary: null metadata pointer");
    if (cdims && product(shape, cdims) == 0) return MTXC_OK;
    if (!r || !a || !b) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary: null buffer");
    ThreadCtx& c = ctx();
    int rc = MTXC_OK;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_broadcast_op<T>(op, r, a, b, cdims, shape, r_strides, a_strides, b_strides, c.sm_count, c.stream());
    });
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE,
                    std::string("mtxc_broadcast_binary: no kernel for dtype ") + dtype_name(dtype));
    return rc;
}
