// The make_pointwise family for sm_100a: greater, less, logical_and, where, floor, full, arctan2,
// arcsin, and the arange generator.
//
// Replaces the Metal branches of those primitives (greater_backend_gpu ... full_backend_gpu,
// Matrix.mm:14281-14440 and the Greater / Less / LogicalAnd / Where / Floor / Full kernels).  The
// metadata is the family's own collapse (make_pointwise, Matrix.mm:13511-13556): the output is
// contiguous and written in order, and each input has one stride array (0 on broadcast axes).  The
// element rules are those of the CPU backends (Matrix.mm:13741-14166):
//   greater / less:  a > b / a < b in the inputs' common dtype -> Bool (NaN compares false)
//   logical_and:     bool(a) && bool(b), inputs already cast to Bool -> Bool
//   where:           cond ? a : b, cond cast to Bool, a and b in their common dtype
//   floor:           float-likes: floor in float, rounded back; integers and Bool: unchanged
//   full:            the (broadcast) value, copied
//   arctan2 / arcsin: inputs cast to Float by the frontend (Matrix.mm:13573-13580), std::atan2 / std::asin
//                    in float (Matrix.mm:13608-13738) -> here CUDA's atan2f / asinf, called, not
//                    restated: within a few ulp of the CPU's libm, not bit-exact
//   arange:          element i = start + i * step in the output dtype: integers as uint64 arithmetic cast
//                    back (wrapping), float-likes as float(start) + float(i) * float(step), each operation
//                    rounded once (no contraction, as the Metal kernel pins with `fp contract(off)`), then
//                    rounded to the dtype (Matrix.mm:14167-14180, ComputeShaders/Arange.metal)
#include "elementwise.cuh"

namespace mtxc {
namespace {

template <typename T>
struct GreaterOp {
    using Out = mbool;
    using In0 = T;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 2;
    __device__ __forceinline__ mbool operator()(T a, T b, T) const { return mbool(less(b, a)); }
};

template <typename T>
struct LessOp {
    using Out = mbool;
    using In0 = T;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 2;
    __device__ __forceinline__ mbool operator()(T a, T b, T) const { return mbool(less(a, b)); }
};

struct LogicalAndOp {
    using Out = mbool;
    using In0 = mbool;
    using In1 = mbool;
    using In2 = mbool;
    static constexpr int kArity = 2;
    __device__ __forceinline__ mbool operator()(mbool a, mbool b, mbool) const {
        return mbool(static_cast<uint8_t>(a) != 0 && static_cast<uint8_t>(b) != 0);
    }
};

template <typename T>
struct WhereOp {
    using Out = T;
    using In0 = mbool;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 3;
    __device__ __forceinline__ T operator()(mbool c, T a, T b) const { return static_cast<uint8_t>(c) != 0 ? a : b; }
};

template <typename T>
struct FloorOp {
    using Out = T;
    using In0 = T;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 1;
    __device__ __forceinline__ T operator()(T x, T, T) const {
        if constexpr (Traits<T>::kFloat) return from_float<T>(floorf(to_float(x)));
        else return x;
    }
};

template <typename T>
struct CopyOp {
    using Out = T;
    using In0 = T;
    using In1 = T;
    using In2 = T;
    static constexpr int kArity = 1;
    __device__ __forceinline__ T operator()(T x, T, T) const { return x; }
};

struct Arctan2Op {
    using Out = float;
    using In0 = float;
    using In1 = float;
    using In2 = float;
    static constexpr int kArity = 2;
    __device__ __forceinline__ float operator()(float a, float b, float) const { return atan2f(a, b); }
};

struct ArcsinOp {
    using Out = float;
    using In0 = float;
    using In1 = float;
    using In2 = float;
    static constexpr int kArity = 1;
    __device__ __forceinline__ float operator()(float x, float, float) const { return asinf(x); }
};

constexpr uint32_t kArity[] = {2, 2, 2, 3, 1, 1, 2, 1};

// arange: element i of the generator (Matrix.mm:14172-14178)
template <typename T>
__device__ __forceinline__ T arange_value(T a, T b, uint64_t i) {
    if constexpr (Traits<T>::kFloat) {
        return from_float<T>(__fadd_rn(to_float(a), __fmul_rn(__ull2float_rn(i), to_float(b))));
    } else {
        return (T)((uint64_t)a + i * (uint64_t)b);
    }
}

// One thread per 16-byte vector of the output (streaming stores); a ragged tail or an output that is not
// 16-byte aligned is written element by element.
template <typename T>
__global__ void __launch_bounds__(256) arange_kernel(T* __restrict__ dst, const T* __restrict__ start,
                                                     const T* __restrict__ step, uint64_t count, bool vec) {
    constexpr int V = Vec16<T>::N;
    const T a = *start, b = *step;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const uint64_t nvec = count / V;
        for (uint64_t v = t; v < nvec; v += stride) {
            Vec16<T> o;
#pragma unroll
            for (int j = 0; j < V; ++j) o.v[j] = arange_value<T>(a, b, v * V + j);
            store_stream(dst + v * V, o);
        }
        for (uint64_t i = nvec * V + t; i < count; i += stride) dst[i] = arange_value<T>(a, b, i);
    } else {
        for (uint64_t i = t; i < count; i += stride) dst[i] = arange_value<T>(a, b, i);
    }
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_pointwise(int op, int dtype, void* dst, const void* const* inputs, uint32_t n_inputs,
                              uint32_t cdims, const uint32_t* shape, const uint32_t* strides) {
    if (int rc = require_init()) return rc;
    if (op < MTXC_PW_GREATER || op > MTXC_PW_ARCSIN) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_pointwise: unknown op");
    if (n_inputs != kArity[op])
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_pointwise: wrong number of inputs for the op");
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_pointwise: cdims > MTXC_MAX_DIMS");
    if (cdims && (!shape || !strides)) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_pointwise: null metadata pointer");
    if (!dst || !inputs) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_pointwise: null buffer");
    for (uint32_t i = 0; i < n_inputs; ++i)
        if (!inputs[i]) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_pointwise: null input buffer");
    if (op == MTXC_PW_LOGICAL_AND && dtype != MTXC_BOOL)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, "mtxc_pointwise: logical_and takes Bool inputs (cast them first)");
    if ((op == MTXC_PW_ARCTAN2 || op == MTXC_PW_ARCSIN) && dtype != MTXC_FLOAT)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, "mtxc_pointwise: arctan2 / arcsin take Float inputs (cast them first)");
    // the output is contiguous: row-major strides of the collapsed shape
    uint32_t sd[MTXC_MAX_DIMS];
    uint64_t acc = 1;
    for (int i = (int)cdims - 1; i >= 0; --i) {
        sd[i] = (uint32_t)acc;
        acc *= shape[i];
    }
    if (cdims && acc > 0xFFFFFFFFull)
        return fail(MTXC_ERR_SHAPE, "mtxc_pointwise: output exceeds 32-bit indexing (as in make_pointwise)");
    ew::MapDesc m{};
    m.dst = dst;
    m.cdims = cdims;
    m.shape = shape;
    m.sd = sd;
    for (uint32_t i = 0; i < n_inputs; ++i) {
        m.src[i] = inputs[i];
        m.ss[i] = strides + (size_t)i * MTXC_MAX_DIMS;
    }
    ThreadCtx& c = ctx();
    const int sms = c.sm_count;
    cudaStream_t s = c.stream();
    int rc = MTXC_OK;
    bool known = true;
    if (op == MTXC_PW_LOGICAL_AND) {
        rc = ew::launch_map<LogicalAndOp>(m, sms, s);
    } else if (op == MTXC_PW_ARCTAN2) {
        rc = ew::launch_map<Arctan2Op>(m, sms, s);
    } else if (op == MTXC_PW_ARCSIN) {
        rc = ew::launch_map<ArcsinOp>(m, sms, s);
    } else {
        known = dispatch_dtype(dtype, [&](auto* tag) {
            using T = std::remove_pointer_t<decltype(tag)>;
            switch (op) {
                case MTXC_PW_GREATER: rc = ew::launch_map<GreaterOp<T>>(m, sms, s); break;
                case MTXC_PW_LESS: rc = ew::launch_map<LessOp<T>>(m, sms, s); break;
                case MTXC_PW_WHERE: rc = ew::launch_map<WhereOp<T>>(m, sms, s); break;
                case MTXC_PW_FLOOR: rc = ew::launch_map<FloorOp<T>>(m, sms, s); break;
                default: rc = ew::launch_map<CopyOp<T>>(m, sms, s); break;
            }
        });
    }
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_pointwise: no kernel for dtype ") + dtype_name(dtype));
    return rc;
}

extern "C" int mtxc_arange(int dtype, void* dst, const void* start, const void* step, uint64_t count) {
    if (int rc = require_init()) return rc;
    if (dtype == MTXC_BOOL) return fail(MTXC_ERR_UNSUPPORTED_DTYPE, "mtxc_arange: arange does not support Bool");
    if (count > 0xFFFFFFFFull) return fail(MTXC_ERR_SHAPE, "mtxc_arange: count exceeds 32-bit indexing (as arange does)");
    if (count == 0) return MTXC_OK;
    if (!dst || !start || !step) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_arange: null buffer");
    ThreadCtx& c = ctx();
    int rc = MTXC_OK;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        constexpr int V = Vec16<T>::N;
        const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
        const uint64_t work = vec ? (count + V - 1) / V : count;
        const uint64_t blocks = std::max<uint64_t>(1, std::min<uint64_t>((work + 255) / 256, (uint64_t)c.sm_count * 16));
        arange_kernel<T><<<(unsigned)blocks, 256, 0, c.stream()>>>(static_cast<T*>(dst), static_cast<const T*>(start),
                                                                   static_cast<const T*>(step), count, vec);
        rc = check_launch("arange_kernel");
    });
    if (!known) return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_arange: no kernel for dtype ") + dtype_name(dtype));
    return rc;
}
