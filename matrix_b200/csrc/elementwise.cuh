// Element-wise map kernels shared by astype / copy, the pointwise family (greater, less,
// logical_and, where, floor, full) and the float unary ops (sqrt, half-precision exp).
//
// An op is a functor with `Out`, `In0..In2`, `kArity` (1..3) and `Out operator()(In0, In1, In2)`.
// The metadata is the reference's: a collapsed shape, the output strides and one stride array per
// input (0 on broadcast axes).  Two kernels:
//
//  * map_rows_kernel: the innermost axis is contiguous in the output and in every input that is not
//    broadcast along it (inner stride 1, or 0 = one value per row).  Work units are row segments;
//    a thread moves chunks of C elements, C = 16 bytes of the smallest operand capped at 64 bytes of
//    the widest, so every access is a 16-byte vector (u8 -> f32 reads 16 B and writes 64 B per chunk)
//    or, for a Bool next to 8-byte types, one 8-byte access.  U chunks are loaded before the first is
//    converted, to keep several loads in flight.
//  * map_generic_kernel: any strides; each thread decodes its element's position from the collapsed
//    shape, innermost axis fastest (32-bit fast division when every index fits in 32 bits).
#pragma once

#include <algorithm>

#include "mtxc_internal.cuh"

namespace mtxc {
namespace ew {

constexpr int kBlock = 256;
constexpr int kMaxIn = 3;
constexpr uint32_t kSegChunks = 2048;  // chunks per work unit (long rows are cut into segments)

template <typename T, int C>
struct alignas(16) Chunk {
    T v[C];
};

// C elements starting at p: one 8-byte access when the chunk is 8 bytes, else C * sizeof(T) / 16
// streaming 16-byte vector accesses (p 16-byte aligned).
template <typename T, int C>
__device__ __forceinline__ void load_chunk(Chunk<T, C>& out, const T* p) {
    constexpr int kBytes = C * (int)sizeof(T);
    static_assert(kBytes == 8 || kBytes % 16 == 0, "chunk must be 8 bytes or whole 16-byte vectors");
    if constexpr (kBytes == 8) {
        uint2 r;
        asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
        memcpy(out.v, &r, 8);
    } else {
#pragma unroll
        for (int i = 0; i < kBytes / 16; ++i) {
            uint4 r;
            asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                : "l"(reinterpret_cast<const char*>(p) + 16 * i));
            memcpy(reinterpret_cast<char*>(out.v) + 16 * i, &r, 16);
        }
    }
}

template <typename T, int C>
__device__ __forceinline__ void store_chunk(T* p, const Chunk<T, C>& in) {
    constexpr int kBytes = C * (int)sizeof(T);
    if constexpr (kBytes == 8) {
        uint2 r;
        memcpy(&r, in.v, 8);
        __stcs(reinterpret_cast<uint2*>(p), r);
    } else {
#pragma unroll
        for (int i = 0; i < kBytes / 16; ++i) {
            uint4 r;
            memcpy(&r, reinterpret_cast<const char*>(in.v) + 16 * i, 16);
            __stcs(reinterpret_cast<uint4*>(reinterpret_cast<char*>(p) + 16 * i), r);
        }
    }
}

template <typename T>
__device__ __forceinline__ T load_elem(const T* p) {
    T out;
    if constexpr (sizeof(T) == 8) {
        unsigned long long r = __ldg(reinterpret_cast<const unsigned long long*>(p));
        memcpy(&out, &r, 8);
    } else if constexpr (sizeof(T) == 4) {
        unsigned int r = __ldg(reinterpret_cast<const unsigned int*>(p));
        memcpy(&out, &r, 4);
    } else if constexpr (sizeof(T) == 2) {
        unsigned short r = __ldg(reinterpret_cast<const unsigned short*>(p));
        memcpy(&out, &r, 2);
    } else {
        unsigned char r = __ldg(reinterpret_cast<const unsigned char*>(p));
        memcpy(&out, &r, 1);
    }
    return out;
}

// Chunk width and unroll depth of an op.
template <class Op>
struct Shape {
    using Out = typename Op::Out;
    static constexpr int kA = Op::kArity;
    static constexpr int kMin0 = (int)std::min(sizeof(Out), sizeof(typename Op::In0));
    static constexpr int kMin1 = kA > 1 ? (int)std::min<size_t>(kMin0, sizeof(typename Op::In1)) : kMin0;
    static constexpr int kMin = kA > 2 ? (int)std::min<size_t>(kMin1, sizeof(typename Op::In2)) : kMin1;
    static constexpr int kMax0 = (int)std::max(sizeof(Out), sizeof(typename Op::In0));
    static constexpr int kMax1 = kA > 1 ? (int)std::max<size_t>(kMax0, sizeof(typename Op::In1)) : kMax0;
    static constexpr int kMax = kA > 2 ? (int)std::max<size_t>(kMax1, sizeof(typename Op::In2)) : kMax1;
    // 16 bytes of the smallest operand, but at most 64 bytes of the widest (so 8-byte types next to
    // Bool move 8 elements per chunk, and the Bool side one 8-byte access)
    static constexpr int C = std::min(16 / kMin, 64 / kMax);
    static constexpr int kInBytes = C * ((int)sizeof(typename Op::In0) + (kA > 1 ? (int)sizeof(typename Op::In1) : 0) +
                                         (kA > 2 ? (int)sizeof(typename Op::In2) : 0));
    static constexpr int kAllBytes = kInBytes + C * (int)sizeof(Out);
    static constexpr int kU0 = std::min(64 / kInBytes, 512 / kAllBytes);
    static constexpr int U = kU0 < 1 ? 1 : (kU0 > 4 ? 4 : kU0);
};

struct RowArgs {
    void* dst;
    const void* src[kMaxIn];
    uint32_t chunks;      // chunks per row
    uint32_t seg_chunks;  // chunks per work unit
    uint32_t segs;        // units per row
    uint32_t units;       // rows * segs (< 2^31)
    uint32_t tpr;         // threads per unit (power of two <= kBlock)
    uint32_t bcast;       // bit k: input k has inner stride 0
    FastDiv seg_div;
    uint32_t n;  // outer axes
    FastDiv fdiv[MTXC_MAX_DIMS];
    uint32_t sd[MTXC_MAX_DIMS];
    uint32_t ss[kMaxIn][MTXC_MAX_DIMS];
};

template <class Op, int C, int U>
__global__ void __launch_bounds__(kBlock) map_rows_kernel(const RowArgs a) {
    using Out = typename Op::Out;
    using I0 = typename Op::In0;
    using I1 = typename Op::In1;
    using I2 = typename Op::In2;
    constexpr int A = Op::kArity;
    const Op op{};
    const uint32_t rpb = kBlock / a.tpr;
    const uint32_t sub = threadIdx.x / a.tpr;
    const uint32_t lane = threadIdx.x % a.tpr;
    const bool b0 = a.bcast & 1u, b1 = a.bcast & 2u, b2 = a.bcast & 4u;
    for (uint32_t u = blockIdx.x * rpb + sub; u < a.units; u += gridDim.x * rpb) {
        uint32_t row = u, seg = 0;
        if (a.segs > 1) a.seg_div.divmod(u, row, seg);
        uint64_t od = 0, o0 = 0, o1 = 0, o2 = 0;
        uint32_t rem = row;
#pragma unroll 1
        for (int i = (int)a.n - 1; i >= 0; --i) {
            uint32_t q, idx;
            a.fdiv[i].divmod(rem, q, idx);
            od += (uint64_t)idx * a.sd[i];
            o0 += (uint64_t)idx * a.ss[0][i];
            if (A > 1) o1 += (uint64_t)idx * a.ss[1][i];
            if (A > 2) o2 += (uint64_t)idx * a.ss[2][i];
            rem = q;
        }
        Out* pd = static_cast<Out*>(a.dst) + od;
        const I0* p0 = static_cast<const I0*>(a.src[0]) + o0;
        const I1* p1 = A > 1 ? static_cast<const I1*>(a.src[1]) + o1 : nullptr;
        const I2* p2 = A > 2 ? static_cast<const I2*>(a.src[2]) + o2 : nullptr;
        // inputs broadcast along the row: one value per row
        const I0 s0 = b0 ? load_elem(p0) : I0{};
        I1 s1{};
        I2 s2{};
        if (A > 1 && b1) s1 = load_elem(p1);
        if (A > 2 && b2) s2 = load_elem(p2);
        const uint32_t c_end = min(a.chunks, (seg + 1) * a.seg_chunks);
        uint32_t c = seg * a.seg_chunks + lane;
        for (; c + (U - 1) * a.tpr < c_end; c += U * a.tpr) {
            Chunk<I0, C> x0[U];
            Chunk<I1, C> x1[U];
            Chunk<I2, C> x2[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const uint64_t e = (uint64_t)(c + j * a.tpr) * C;
                if (!b0) load_chunk(x0[j], p0 + e);
                if (A > 1 && !b1) load_chunk(x1[j], p1 + e);
                if (A > 2 && !b2) load_chunk(x2[j], p2 + e);
            }
#pragma unroll
            for (int j = 0; j < U; ++j) {
                Chunk<Out, C> y;
#pragma unroll
                for (int k = 0; k < C; ++k)
                    y.v[k] = op(b0 ? s0 : x0[j].v[k], (A > 1 && !b1) ? x1[j].v[k] : s1, (A > 2 && !b2) ? x2[j].v[k] : s2);
                store_chunk(pd + (uint64_t)(c + j * a.tpr) * C, y);
            }
        }
        for (; c < c_end; c += a.tpr) {
            const uint64_t e = (uint64_t)c * C;
            Chunk<I0, C> x0;
            Chunk<I1, C> x1;
            Chunk<I2, C> x2;
            if (!b0) load_chunk(x0, p0 + e);
            if (A > 1 && !b1) load_chunk(x1, p1 + e);
            if (A > 2 && !b2) load_chunk(x2, p2 + e);
            Chunk<Out, C> y;
#pragma unroll
            for (int k = 0; k < C; ++k)
                y.v[k] = op(b0 ? s0 : x0.v[k], (A > 1 && !b1) ? x1.v[k] : s1, (A > 2 && !b2) ? x2.v[k] : s2);
            store_chunk(pd + e, y);
        }
    }
}

struct GenericArgs {
    void* dst;
    const void* src[kMaxIn];
    uint64_t total;
    uint32_t n;  // all axes
    uint32_t shape[MTXC_MAX_DIMS];
    FastDiv fdiv[MTXC_MAX_DIMS];
    uint32_t sd[MTXC_MAX_DIMS];
    uint32_t ss[kMaxIn][MTXC_MAX_DIMS];
};

template <class Op, bool k32>
__global__ void __launch_bounds__(kBlock) map_generic_kernel(const GenericArgs g) {
    using Out = typename Op::Out;
    using I0 = typename Op::In0;
    using I1 = typename Op::In1;
    using I2 = typename Op::In2;
    constexpr int A = Op::kArity;
    const Op op{};
    for (uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < g.total;
         gid += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t od = 0, o0 = 0, o1 = 0, o2 = 0;
        if constexpr (k32) {
            uint32_t rem = (uint32_t)gid;
#pragma unroll 1
            for (int i = (int)g.n - 1; i >= 0; --i) {
                uint32_t q, idx;
                g.fdiv[i].divmod(rem, q, idx);
                od += (uint64_t)idx * g.sd[i];
                o0 += (uint64_t)idx * g.ss[0][i];
                if (A > 1) o1 += (uint64_t)idx * g.ss[1][i];
                if (A > 2) o2 += (uint64_t)idx * g.ss[2][i];
                rem = q;
            }
        } else {
            uint64_t rem = gid;
#pragma unroll 1
            for (int i = (int)g.n - 1; i >= 0; --i) {
                const uint64_t idx = rem % g.shape[i];
                od += idx * g.sd[i];
                o0 += idx * g.ss[0][i];
                if (A > 1) o1 += idx * g.ss[1][i];
                if (A > 2) o2 += idx * g.ss[2][i];
                rem /= g.shape[i];
            }
        }
        const I0 x0 = load_elem(static_cast<const I0*>(g.src[0]) + o0);
        I1 x1{};
        I2 x2{};
        if (A > 1) x1 = load_elem(static_cast<const I1*>(g.src[1]) + o1);
        if (A > 2) x2 = load_elem(static_cast<const I2*>(g.src[2]) + o2);
        static_cast<Out*>(g.dst)[od] = op(x0, x1, x2);
    }
}

// Host-side description of one map launch (reference metadata, not yet validated for the row path).
struct MapDesc {
    void* dst;
    const void* src[kMaxIn];
    uint32_t cdims;
    const uint32_t* shape;
    const uint32_t* sd;
    const uint32_t* ss[kMaxIn];
};

// Launches the row kernel when the innermost axis allows 16-byte chunks, else the generic kernel.
template <class Op>
int launch_map(const MapDesc& m, int sm_count, cudaStream_t stream) {
    using S = Shape<Op>;
    constexpr int A = Op::kArity;
    constexpr int C = S::C;
    const size_t in_size[kMaxIn] = {sizeof(typename Op::In0), sizeof(typename Op::In1), sizeof(typename Op::In2)};
    uint32_t one = 1, zero = 0;
    uint32_t cdims = m.cdims;
    const uint32_t* shape = m.shape;
    const uint32_t* sd = m.sd;
    const uint32_t* ss[kMaxIn] = {m.ss[0], m.ss[1], m.ss[2]};
    if (cdims == 0) {  // one element at offset 0 of every operand
        cdims = 1;
        shape = &one;
        sd = &one;
        for (int i = 0; i < kMaxIn; ++i) ss[i] = &zero;
    }
    const uint64_t total = product(shape, cdims);
    if (total == 0) return MTXC_OK;
    const uint32_t k = cdims - 1;
    bool rows_ok = sd[k] == 1 && shape[k] % C == 0 && aligned16(m.dst);
    uint32_t bcast = 0;
    for (int i = 0; i < A && rows_ok; ++i) {
        if (ss[i][k] == 0) bcast |= 1u << i;
        else rows_ok = ss[i][k] == 1 && aligned16(m.src[i]);
    }
    const uint32_t chunks = shape[k] / C;
    uint32_t seg_chunks = std::min<uint32_t>(std::max<uint32_t>(chunks, 1), kSegChunks);
    const uint32_t segs = (chunks + seg_chunks - 1) / std::max<uint32_t>(seg_chunks, 1);
    const uint64_t rows = total / shape[k];
    rows_ok = rows_ok && chunks > 0 && rows * segs < (1ull << 31);
    for (uint32_t j = 0; j < k && rows_ok; ++j) {
        if (shape[j] == 1) continue;
        rows_ok = shape[j] < (1u << 31) && (uint64_t)sd[j] * sizeof(typename Op::Out) % 16 == 0;
        for (int i = 0; i < A && rows_ok; ++i)
            rows_ok = (bcast >> i & 1u) ? true : (uint64_t)ss[i][j] * in_size[i] % 16 == 0;
    }
    if (rows_ok) {
        RowArgs a{};
        a.dst = m.dst;
        for (int i = 0; i < kMaxIn; ++i) a.src[i] = i < A ? m.src[i] : nullptr;
        a.chunks = chunks;
        a.seg_chunks = seg_chunks;
        a.segs = segs;
        a.seg_div = FastDiv(segs);
        a.units = (uint32_t)(rows * segs);
        uint32_t tpr = 1;
        while (tpr < seg_chunks && tpr < (uint32_t)kBlock) tpr <<= 1;
        a.tpr = tpr;
        a.bcast = bcast;
        a.n = k;
        for (uint32_t j = 0; j < k; ++j) {
            a.fdiv[j] = FastDiv(shape[j]);
            a.sd[j] = sd[j];
            for (int i = 0; i < A; ++i) a.ss[i][j] = ss[i][j];
        }
        const uint32_t rpb = kBlock / tpr;
        const uint64_t blocks = std::min<uint64_t>((a.units + rpb - 1) / rpb, (uint64_t)sm_count * 4);
        map_rows_kernel<Op, C, S::U><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        return check_launch("map_rows_kernel");
    }
    GenericArgs g{};
    g.dst = m.dst;
    for (int i = 0; i < kMaxIn; ++i) g.src[i] = i < A ? m.src[i] : nullptr;
    g.total = total;
    g.n = cdims;
    bool k32 = total < (1ull << 32);
    for (uint32_t j = 0; j < cdims; ++j) {
        g.shape[j] = shape[j];
        k32 = k32 && shape[j] < (1u << 31);
        g.fdiv[j] = FastDiv(shape[j] < (1u << 31) ? shape[j] : 1u);
        g.sd[j] = sd[j];
        for (int i = 0; i < A; ++i) g.ss[i][j] = ss[i][j];
    }
    const uint64_t blocks = std::min<uint64_t>((total + kBlock - 1) / kBlock, (uint64_t)sm_count * 16);
    if (k32) map_generic_kernel<Op, true><<<(unsigned)blocks, kBlock, 0, stream>>>(g);
    else map_generic_kernel<Op, false><<<(unsigned)blocks, kBlock, 0, stream>>>(g);
    return check_launch("map_generic_kernel");
}

}  // namespace ew
}  // namespace mtxc
