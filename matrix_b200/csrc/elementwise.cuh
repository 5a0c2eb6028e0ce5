// Element-wise map kernels shared by astype / copy, the pointwise family (greater, less,
// logical_and, where, floor, full) and the float unary ops (sqrt, half-precision exp).
//
// An op is a functor with `Out`, `In0..In2`, `kArity` (1..3) and `Out operator()(In0, In1, In2)`.
// The metadata is the reference's: a collapsed shape, the output strides and one stride array per
// input (0 on broadcast axes).  Two kernels:
//
//  * map_rows_kernel: the innermost axis is contiguous in the output and in every input that is not
//    broadcast along it (inner stride 1, or 0 = one value per row).  Work units are row segments cut
//    into slots of W elements, W * (widest element size) = 16 bytes; lanes take consecutive slots, so
//    each access of each operand is contiguous across the warp (u8 -> f32: 4-byte loads and 16-byte
//    stores, both covering 512 contiguous bytes per warp instruction).  U slots are loaded before the
//    first is converted, about 128 bytes of loads in flight per thread.
//  * map_generic_kernel: any strides; each thread decodes its element's position from the collapsed
//    shape, innermost axis fastest (32-bit fast division when every index fits in 32 bits).
#pragma once

#include <algorithm>

#include "mtxc_internal.cuh"

namespace mtxc {
namespace ew {

constexpr int kBlock = 256;
constexpr int kMaxIn = 3;
constexpr uint32_t kSegSlots = 4096;  // slots per work unit (long rows are cut into segments)

// A slot: W consecutive elements of one operand, moved with one access of W * sizeof(T) bytes
// (2, 4, 8 or 16).  Lanes of a warp take consecutive slots, so every operand's access is contiguous
// across the warp whatever its element size.
template <typename T, int W>
struct alignas(W * sizeof(T)) Slot {
    T v[W];
};

template <typename T, int W>
__device__ __forceinline__ void load_slot(Slot<T, W>& out, const T* p) {
    constexpr int kBytes = W * (int)sizeof(T);
    if constexpr (kBytes == 16) {
        uint4 r;
        asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
            : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
            : "l"(p));
        memcpy(out.v, &r, 16);
    } else if constexpr (kBytes == 8) {
        uint2 r;
        asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
        memcpy(out.v, &r, 8);
    } else if constexpr (kBytes == 4) {
        unsigned r;
        asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
        memcpy(out.v, &r, 4);
    } else {
        static_assert(kBytes == 2, "slot of 2, 4, 8 or 16 bytes");
        unsigned short r;
        asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
        memcpy(out.v, &r, 2);
    }
}

template <typename T, int W>
__device__ __forceinline__ void store_slot(T* p, const Slot<T, W>& in) {
    constexpr int kBytes = W * (int)sizeof(T);
    if constexpr (kBytes == 16) {
        uint4 r;
        memcpy(&r, in.v, 16);
        __stcs(reinterpret_cast<uint4*>(p), r);
    } else if constexpr (kBytes == 8) {
        uint2 r;
        memcpy(&r, in.v, 8);
        __stcs(reinterpret_cast<uint2*>(p), r);
    } else if constexpr (kBytes == 4) {
        unsigned r;
        memcpy(&r, in.v, 4);
        __stcs(reinterpret_cast<unsigned*>(p), r);
    } else {
        unsigned short r;
        memcpy(&r, in.v, 2);
        __stcs(reinterpret_cast<unsigned short*>(p), r);
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

// Slot width and unroll depth of an op: a slot is 16 bytes of the widest operand; U slots per thread
// per iteration are loaded before the first is converted, about 128 bytes of loads in flight.
template <class Op>
struct Shape {
    using Out = typename Op::Out;
    static constexpr int kA = Op::kArity;
    static constexpr int kMax0 = (int)std::max(sizeof(Out), sizeof(typename Op::In0));
    static constexpr int kMax1 = kA > 1 ? (int)std::max<size_t>(kMax0, sizeof(typename Op::In1)) : kMax0;
    static constexpr int kMax = kA > 2 ? (int)std::max<size_t>(kMax1, sizeof(typename Op::In2)) : kMax1;
    static constexpr int W = 16 / kMax;
    static constexpr int kInBytes = W * ((int)sizeof(typename Op::In0) + (kA > 1 ? (int)sizeof(typename Op::In1) : 0) +
                                         (kA > 2 ? (int)sizeof(typename Op::In2) : 0));
    static constexpr int kU0 = 128 / kInBytes;
    static constexpr int U = kU0 < 1 ? 1 : (kU0 > 16 ? 16 : kU0);
};

struct RowArgs {
    void* dst;
    const void* src[kMaxIn];
    uint32_t slots;      // slots per row
    uint32_t seg_slots;  // slots per work unit
    uint32_t segs;       // units per row
    uint32_t units;      // rows * segs (< 2^31)
    uint32_t tpr;        // threads per unit (power of two <= kBlock)
    uint32_t bcast;      // bit k: input k has inner stride 0
    FastDiv seg_div;
    uint32_t n;  // outer axes
    FastDiv fdiv[MTXC_MAX_DIMS];
    uint32_t sd[MTXC_MAX_DIMS];
    uint32_t ss[kMaxIn][MTXC_MAX_DIMS];
};

template <class Op, int W, int U>
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
        const uint32_t c_end = min(a.slots, (seg + 1) * a.seg_slots);
        uint32_t c = seg * a.seg_slots + lane;
        for (; c + (U - 1) * a.tpr < c_end; c += U * a.tpr) {
            Slot<I0, W> x0[U];
            Slot<I1, W> x1[U];
            Slot<I2, W> x2[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const uint64_t e = (uint64_t)(c + j * a.tpr) * W;
                if (!b0) load_slot(x0[j], p0 + e);
                if (A > 1 && !b1) load_slot(x1[j], p1 + e);
                if (A > 2 && !b2) load_slot(x2[j], p2 + e);
            }
#pragma unroll
            for (int j = 0; j < U; ++j) {
                Slot<Out, W> y;
#pragma unroll
                for (int k = 0; k < W; ++k)
                    y.v[k] = op(b0 ? s0 : x0[j].v[k], (A > 1 && !b1) ? x1[j].v[k] : s1, (A > 2 && !b2) ? x2[j].v[k] : s2);
                store_slot(pd + (uint64_t)(c + j * a.tpr) * W, y);
            }
        }
        for (; c < c_end; c += a.tpr) {
            const uint64_t e = (uint64_t)c * W;
            Slot<I0, W> x0;
            Slot<I1, W> x1;
            Slot<I2, W> x2;
            if (!b0) load_slot(x0, p0 + e);
            if (A > 1 && !b1) load_slot(x1, p1 + e);
            if (A > 2 && !b2) load_slot(x2, p2 + e);
            Slot<Out, W> y;
#pragma unroll
            for (int k = 0; k < W; ++k)
                y.v[k] = op(b0 ? s0 : x0.v[k], (A > 1 && !b1) ? x1.v[k] : s1, (A > 2 && !b2) ? x2.v[k] : s2);
            store_slot(pd + e, y);
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

// Launches the row kernel when the innermost axis allows whole slots, else the generic kernel.
template <class Op>
int launch_map(const MapDesc& m, int sm_count, cudaStream_t stream) {
    using S = Shape<Op>;
    constexpr int A = Op::kArity;
    constexpr int W = S::W;
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
    auto aligned = [](const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; };
    bool rows_ok = sd[k] == 1 && shape[k] % W == 0 && aligned(m.dst, W * sizeof(typename Op::Out));
    uint32_t bcast = 0;
    for (int i = 0; i < A && rows_ok; ++i) {
        if (ss[i][k] == 0) bcast |= 1u << i;
        else rows_ok = ss[i][k] == 1 && aligned(m.src[i], W * in_size[i]);
    }
    const uint32_t slots = shape[k] / W;
    const uint32_t seg_slots = std::min<uint32_t>(std::max<uint32_t>(slots, 1), kSegSlots);
    const uint32_t segs = (slots + seg_slots - 1) / seg_slots;
    const uint64_t rows = total / shape[k];
    rows_ok = rows_ok && slots > 0 && rows * segs < (1ull << 31);
    for (uint32_t j = 0; j < k && rows_ok; ++j) {
        if (shape[j] == 1) continue;
        rows_ok = shape[j] < (1u << 31) && sd[j] % W == 0;
        for (int i = 0; i < A && rows_ok; ++i) rows_ok = (bcast >> i & 1u) || ss[i][j] % W == 0;
    }
    if (rows_ok) {
        RowArgs a{};
        a.dst = m.dst;
        for (int i = 0; i < kMaxIn; ++i) a.src[i] = i < A ? m.src[i] : nullptr;
        a.slots = slots;
        a.seg_slots = seg_slots;
        a.segs = segs;
        a.seg_div = FastDiv(segs);
        a.units = (uint32_t)(rows * segs);
        uint32_t tpr = 1;
        while (tpr < seg_slots && tpr < (uint32_t)kBlock) tpr <<= 1;
        a.tpr = tpr;
        a.bcast = bcast;
        a.n = k;
        for (uint32_t j = 0; j < k; ++j) {
            a.fdiv[j] = FastDiv(shape[j]);
            a.sd[j] = sd[j];
            for (int i = 0; i < A; ++i) a.ss[i][j] = ss[i][j];
        }
        // one block per rpb work units: measured on B200 against grids of 2-64 blocks per SM looping over
        // the units, the hardware block scheduler balances best (u8 -> f32 astype 0.83 -> 0.98 of the
        // measured copy bandwidth, where 0.82 -> 0.98)
        const uint32_t rpb = kBlock / tpr;
        const uint64_t blocks = (a.units + rpb - 1) / rpb;
        map_rows_kernel<Op, W, S::U><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
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
