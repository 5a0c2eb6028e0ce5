// Elementwise unary ops for sm_100a: exp (ExpPrimitive, primitives.cpp:5332-5463) and sqrt
// (SqrtPrimitive).
//
// Replaces ComputeShaders/exp.metal and sqrt.metal behind matrix::exp / matrix::sqrt(output, dev)
// (Matrix.mm:6949-7011, 6813-6867).  Both ops take Float or Float16 (the frontends promote every other
// dtype first: promote_types(type, Float16), Matrix.mm:6798-6811, 6934-6947).  The metadata is the
// primitive's collapse_dims(shape, output strides, input strides); the element position is decoded
// from the collapsed shape, innermost axis fastest, as the CPU branches do (Matrix.mm:6870-6925,
// 7014-7063).  exp is CUDA's expf (full-range, <= 2 ulp), so results agree with the CPU's std::exp
// within a few ulp rather than bit for bit; Float16 exp rounds that float result once.  sqrt is the
// IEEE correctly rounded square root (sqrtf), bit-exact with std::sqrt; for Float16 the float root
// rounded once is the correctly rounded half result.
#include <algorithm>

#include "elementwise.cuh"

namespace mtxc {
namespace {

constexpr int kBlock = 256;
constexpr uint32_t kSegVecs = 4096;

struct UnaryRows {
    float* dst;
    const float* src;
    uint32_t rows;
    uint32_t vec_per_row;
    uint32_t seg_vecs;  // vectors per work unit (rows are cut into segments of this size)
    uint32_t segs;      // segments per row
    uint32_t units;     // rows * segs (< 2^31)
    uint32_t tpr;
    FastDiv seg_div;    // divides a unit index by segs
    Dims d;  // outer axes: shape (fast divisors), dst strides in s0, src strides in s1
};

__global__ void __launch_bounds__(kBlock) exp_rows_kernel(const UnaryRows a) {
    const uint32_t rows_per_block = kBlock / a.tpr;
    const uint32_t sub = threadIdx.x / a.tpr;
    const uint32_t lane = threadIdx.x % a.tpr;
    for (uint32_t u = blockIdx.x * rows_per_block + sub; u < a.units; u += gridDim.x * rows_per_block) {
        uint32_t row = u, seg = 0;
        if (a.segs > 1) a.seg_div.divmod(u, row, seg);
        const uint32_t c_end = min(a.vec_per_row, (seg + 1) * a.seg_vecs);
        uint64_t od = 0, os = 0;
        uint32_t rem = row;
#pragma unroll 1
        for (int i = (int)a.d.n - 1; i >= 0; --i) {
            uint32_t q, idx;
            a.d.fdiv[i].divmod(rem, q, idx);
            od += (uint64_t)idx * a.d.s0[i];
            os += (uint64_t)idx * a.d.s1[i];
            rem = q;
        }
        const float* ps = a.src + os;
        float* pd = a.dst + od;
        uint32_t c = seg * a.seg_vecs + lane;
        // four loads in flight per thread before the first is used
        for (; c + 3 * a.tpr < c_end; c += 4 * a.tpr) {
            Vec16<float> x[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) x[k] = load_stream(ps + (uint64_t)(c + k * a.tpr) * 4);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
#pragma unroll
                for (int j = 0; j < 4; ++j) x[k].v[j] = expf(x[k].v[j]);
                store_stream(pd + (uint64_t)(c + k * a.tpr) * 4, x[k]);
            }
        }
        for (; c < c_end; c += a.tpr) {
            Vec16<float> x = load_stream(ps + (uint64_t)c * 4);
#pragma unroll
            for (int j = 0; j < 4; ++j) x.v[j] = expf(x.v[j]);
            store_stream(pd + (uint64_t)c * 4, x);
        }
    }
}

struct UnaryGeneric {
    float* dst;
    const float* src;
    uint64_t total;
    uint32_t cdims;
    uint32_t shape[MTXC_MAX_DIMS];
    uint32_t sd[MTXC_MAX_DIMS];
    uint32_t ss[MTXC_MAX_DIMS];
};

__global__ void __launch_bounds__(kBlock) exp_generic_kernel(const UnaryGeneric g) {
    for (uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < g.total;
         gid += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t od = 0, os = 0, rem = gid;
        for (int i = (int)g.cdims - 1; i >= 0; --i) {
            const uint64_t idx = rem % g.shape[i];
            od += idx * g.sd[i];
            os += idx * g.ss[i];
            rem /= g.shape[i];
        }
        g.dst[od] = expf(g.src[os]);
    }
}

int launch_exp(float* dst, const float* src, uint32_t cdims, const uint32_t* shape, const uint32_t* sd,
               const uint32_t* ss, int sm_count, cudaStream_t stream) {
    uint32_t one = 1;
    if (cdims == 0) {
        cdims = 1;
        shape = sd = ss = &one;
    }
    const uint64_t total = product(shape, cdims);
    if (total == 0) return MTXC_OK;
    const uint32_t k = cdims - 1;
    bool rows_ok = sd[k] == 1 && ss[k] == 1 && shape[k] % 4 == 0 && aligned16(dst) && aligned16(src) &&
                   (total / shape[k]) * ((shape[k] / 4 + kSegVecs - 1) / kSegVecs) < (1ull << 31);
    for (uint32_t i = 0; i < k && rows_ok; ++i) rows_ok = shape[i] == 1 || (sd[i] % 4 == 0 && ss[i] % 4 == 0);
    if (rows_ok) {
        UnaryRows a{};
        a.dst = dst;
        a.src = src;
        a.rows = (uint32_t)(total / shape[k]);
        a.vec_per_row = shape[k] / 4;
        a.seg_vecs = std::min<uint32_t>(a.vec_per_row, kSegVecs);
        a.segs = (a.vec_per_row + a.seg_vecs - 1) / a.seg_vecs;
        a.seg_div = FastDiv(a.segs);
        uint32_t tpr = 1;
        while (tpr < a.seg_vecs && tpr < (uint32_t)kBlock) tpr <<= 1;
        a.tpr = tpr;
        a.d.n = k;
        for (uint32_t i = 0; i < k; ++i) {
            a.d.shape[i] = shape[i];
            a.d.s0[i] = sd[i];
            a.d.s1[i] = ss[i];
            a.d.fdiv[i] = FastDiv(shape[i]);
        }
        const uint32_t rpb = kBlock / tpr;
        const uint64_t units = (uint64_t)a.rows * a.segs;
        a.units = (uint32_t)units;
        const uint64_t blocks = std::min<uint64_t>((units + rpb - 1) / rpb, (uint64_t)sm_count * 8);
        exp_rows_kernel<<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        return check_launch("exp_rows_kernel");
    }
    UnaryGeneric g{};
    g.dst = dst;
    g.src = src;
    g.total = total;
    g.cdims = cdims;
    for (uint32_t i = 0; i < cdims; ++i) {
        g.shape[i] = shape[i];
        g.sd[i] = sd[i];
        g.ss[i] = ss[i];
    }
    const uint64_t blocks = std::min<uint64_t>((total + kBlock - 1) / kBlock, (uint64_t)sm_count * 16);
    exp_generic_kernel<<<(unsigned)blocks, kBlock, 0, stream>>>(g);
    return check_launch("exp_generic_kernel");
}

template <typename T>
struct ExpOp {
    using Out = T;
    using In0 = T;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 1;
    __device__ __forceinline__ T operator()(T x, T, T) const { return from_float<T>(expf(to_float(x))); }
};

template <typename T>
struct SqrtOp {
    using Out = T;
    using In0 = T;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 1;
    __device__ __forceinline__ T operator()(T x, T, T) const { return from_float<T>(sqrtf(to_float(x))); }
};

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_unary(int op, int dtype, void* dst, const void* src, uint32_t cdims, const uint32_t* shape,
                          const uint32_t* dst_strides, const uint32_t* src_strides) {
    if (int rc = require_init()) return rc;
    if (op != MTXC_UNARY_EXP && op != MTXC_UNARY_SQRT) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_unary: unknown op");
    if (dtype != MTXC_FLOAT && dtype != MTXC_FLOAT16)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_unary: no kernel for dtype ") + dtype_name(dtype) +
                                                    " (exp and sqrt take Float or Float16)");
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_unary: cdims > MTXC_MAX_DIMS");
    if (cdims && (!shape || !dst_strides || !src_strides))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_unary: null metadata pointer");
    if (cdims && product(shape, cdims) == 0) return MTXC_OK;
    if (!dst || !src) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_unary: null buffer");
    ThreadCtx& c = ctx();
    if (op == MTXC_UNARY_EXP && dtype == MTXC_FLOAT)
        return launch_exp(static_cast<float*>(dst), static_cast<const float*>(src), cdims, shape, dst_strides,
                          src_strides, c.sm_count, c.stream());
    ew::MapDesc m{};
    m.dst = dst;
    m.src[0] = src;
    m.cdims = cdims;
    m.shape = shape;
    m.sd = dst_strides;
    m.ss[0] = src_strides;
    if (op == MTXC_UNARY_EXP) return ew::launch_map<ExpOp<__half>>(m, c.sm_count, c.stream());
    if (dtype == MTXC_FLOAT) return ew::launch_map<SqrtOp<float>>(m, c.sm_count, c.stream());
    return ew::launch_map<SqrtOp<__half>>(m, c.sm_count, c.stream());
}
