// Fused row softmax for sm_100a: the reference's compiled trace
//     m = x.max(-1, true); e = matrix::exp(x - m); y = e / e.sum(-1, true)
// (MaxReductionPrimitive, SubtractionPrimitive, ExpPrimitive, SumPrimitive, DivisionPrimitive;
// benchmark config 5a) evaluated in one kernel that reads x once and writes y once, instead of the
// five kernels and ~4 passes over the data the trace takes one primitive at a time.
//
// Each row is held by one thread-block cluster: C CTAs of 256 threads, each thread keeping 4 * VPT
// elements in registers.  The row maximum and the row sum are reduced per warp (shuffles), per CTA
// (shared memory) and across the cluster through distributed shared memory: each CTA pushes its
// partial into a slot of every CTA of the cluster, one cluster barrier later each CTA combines the C
// slots in rank order from its own shared memory, so all CTAs of a row agree on m and s.  A first
// cluster barrier (arrive at entry, wait before the first push) guarantees every peer CTA is running
// before its shared memory is written.
//
// Arithmetic follows the trace element by element: m is the reference Max (start from -FLT_MAX, an
// element replaces it only when strictly greater, so NaN never wins); t = x - m and e = expf(t) are
// the same single operations the Sub and Exp primitives perform.  Two steps differ: the fp32
// additions of s run in a tree instead of the Sum primitive's sequential loop, and y = e * (1 / s)
// with one correctly rounded reciprocal per row replaces the Div primitive's e / s (within 1 ulp of
// it; the division was a third of the kernel's instructions).  (The
// sign of a zero maximum cannot matter: exp(x - (+0)) and exp(x - (-0)) are equal for every x.)
#include <algorithm>

#include <cooperative_groups.h>

#include "mtxc_internal.cuh"

namespace cg = cooperative_groups;

namespace mtxc {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, v, m);
        v = (v < o) ? o : v;
    }
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

// Cluster-wide barrier in which only the warp that wrote other CTAs' shared memory arrives with release
// semantics; the other warps arrive relaxed (they published nothing, and a release arrival fences each
// warp's prior memory operations).  Every thread waits with acquire semantics, so the released writes
// are visible to all readers after it.  `writer` must be uniform across the warp (.aligned).
__device__ __forceinline__ void cluster_barrier(bool writer) {
    if (writer) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    else asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// FULL: the row fills the cluster exactly (row_len == C * 256 * 4 * VPT), so no vector needs a bounds
// predicate.
template <int C, int VPT, bool FULL>
__global__ void __cluster_dims__(C, 1, 1) __launch_bounds__(kThreads)
    softmax_rows_kernel(float* __restrict__ dst, const float* __restrict__ src, uint32_t row_len,
                        uint64_t src_row_stride, uint64_t dst_row_stride) {
    __shared__ float warp_part[kThreads / 32];
    // per-CTA partials of the cluster, pushed here by every CTA of the row (slot = sender's rank)
    __shared__ float max_slot[C];
    __shared__ float sum_slot[C];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    const uint64_t row = blockIdx.x / C;
    const float* x = src + row * src_row_stride;
    float* y = dst + row * dst_row_stride;
    const uint32_t nvec = row_len / 4;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // vectors of this thread: rank * (256 * VPT) + k * 256 + threadIdx.x, k < VPT (coalesced per k)
    // all VPT loads are issued before any is used, so each thread keeps VPT 16-byte loads in flight
    float4 v[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t c = rank * (kThreads * VPT) + k * kThreads + threadIdx.x;
        if (FULL || c < nvec) {
            const Vec16<float> t = load_stream(x + (uint64_t)c * 4);
            v[k] = make_float4(t.v[0], t.v[1], t.v[2], t.v[3]);
        } else {
            v[k] = make_float4(lowest_value<float>(), lowest_value<float>(), lowest_value<float>(),
                               lowest_value<float>());
        }
    }
    // Distributed shared memory may be written only once every CTA of the cluster is known to be
    // running.  Every thread arrives here, with its loads still in flight (relaxed: nothing to publish
    // yet), and waits just before the first push into a peer CTA's shared memory below.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    float m = lowest_value<float>();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        m = (m < v[k].x) ? v[k].x : m;
        m = (m < v[k].y) ? v[k].y : m;
        m = (m < v[k].z) ? v[k].z : m;
        m = (m < v[k].w) ? v[k].w : m;
    }
    m = warp_max(m);
    if (lane == 0) warp_part[warp] = m;
    __syncthreads();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA of the cluster has started
    if (warp == 0) {
        float w = lane < kThreads / 32 ? warp_part[lane] : lowest_value<float>();
        w = warp_max(w);
        // push this CTA's maximum into slot `rank` of every CTA of the cluster (lanes 0..C-1)
        if (lane < C) *cluster.map_shared_rank(&max_slot[rank], lane) = w;
    }
    // every CTA's pushes are complete and visible after this barrier; afterwards a CTA reads only its
    // own shared memory, so no CTA can leave while another still reads from it
    cluster_barrier(warp == 0);
    m = lowest_value<float>();
#pragma unroll
    for (int r = 0; r < C; ++r) m = (m < max_slot[r]) ? max_slot[r] : m;

    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t c = rank * (kThreads * VPT) + k * kThreads + threadIdx.x;
        if (FULL || c < nvec) {
            v[k].x = expf(__fsub_rn(v[k].x, m));
            v[k].y = expf(__fsub_rn(v[k].y, m));
            v[k].z = expf(__fsub_rn(v[k].z, m));
            v[k].w = expf(__fsub_rn(v[k].w, m));
            s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[k].x, v[k].y), __fadd_rn(v[k].z, v[k].w)));
        }
    }
    s = warp_sum(s);
    __syncthreads();  // warp_part is reused
    if (lane == 0) warp_part[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float w = lane < kThreads / 32 ? warp_part[lane] : 0.0f;
        w = warp_sum(w);
        if (lane < C) *cluster.map_shared_rank(&sum_slot[rank], lane) = w;
    }
    cluster_barrier(warp == 0);
    s = 0.0f;
#pragma unroll
    for (int r = 0; r < C; ++r) s = __fadd_rn(s, sum_slot[r]);
    const float inv = __frcp_rn(s);  // e * (1 / s): within 1 ulp of e / s, a quarter of the instructions

#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t c = rank * (kThreads * VPT) + k * kThreads + threadIdx.x;
        if (FULL || c < nvec) {
            Vec16<float> o;
            o.v[0] = __fmul_rn(v[k].x, inv);
            o.v[1] = __fmul_rn(v[k].y, inv);
            o.v[2] = __fmul_rn(v[k].z, inv);
            o.v[3] = __fmul_rn(v[k].w, inv);
            store_stream(y + (uint64_t)c * 4, o);
        }
    }
}

// Rows of at most 32 * 4 * VPL elements: one warp per row, no shared memory, grid-stride over rows.
template <int VPL>
__global__ void __launch_bounds__(kThreads) softmax_warp_rows_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                                                   uint64_t rows, uint32_t row_len, uint64_t src_row_stride,
                                                                   uint64_t dst_row_stride) {
    const uint32_t lane = threadIdx.x % 32;
    const uint64_t warps = (uint64_t)gridDim.x * (kThreads / 32);
    const uint32_t nvec = row_len / 4;
    for (uint64_t row = (uint64_t)blockIdx.x * (kThreads / 32) + threadIdx.x / 32; row < rows; row += warps) {
        const float* x = src + row * src_row_stride;
        float* y = dst + row * dst_row_stride;
        float4 v[VPL];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const uint32_t c = k * 32 + lane;
            if (c < nvec) {
                const Vec16<float> t = load_stream(x + (uint64_t)c * 4);
                v[k] = make_float4(t.v[0], t.v[1], t.v[2], t.v[3]);
            } else {
                v[k] = make_float4(lowest_value<float>(), lowest_value<float>(), lowest_value<float>(),
                                   lowest_value<float>());
            }
        }
        float m = lowest_value<float>();
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            m = (m < v[k].x) ? v[k].x : m;
            m = (m < v[k].y) ? v[k].y : m;
            m = (m < v[k].z) ? v[k].z : m;
            m = (m < v[k].w) ? v[k].w : m;
        }
        m = warp_max(m);
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if (k * 32 + lane < nvec) {
                v[k].x = expf(__fsub_rn(v[k].x, m));
                v[k].y = expf(__fsub_rn(v[k].y, m));
                v[k].z = expf(__fsub_rn(v[k].z, m));
                v[k].w = expf(__fsub_rn(v[k].w, m));
                s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[k].x, v[k].y), __fadd_rn(v[k].z, v[k].w)));
            }
        }
        s = warp_sum(s);
        const float inv = __frcp_rn(s);
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const uint32_t c = k * 32 + lane;
            if (c < nvec) {
                Vec16<float> o;
                o.v[0] = __fmul_rn(v[k].x, inv);
                o.v[1] = __fmul_rn(v[k].y, inv);
                o.v[2] = __fmul_rn(v[k].z, inv);
                o.v[3] = __fmul_rn(v[k].w, inv);
                store_stream(y + (uint64_t)c * 4, o);
            }
        }
    }
}

template <int VPL>
int launch_softmax_warps(float* dst, const float* src, uint64_t rows, uint32_t len, uint64_t ss, uint64_t ds,
                         int sm_count, cudaStream_t stream) {
    const uint64_t blocks = std::min<uint64_t>((rows + kThreads / 32 - 1) / (kThreads / 32), (uint64_t)sm_count * 16);
    softmax_warp_rows_kernel<VPL><<<(unsigned)blocks, kThreads, 0, stream>>>(dst, src, rows, len, ss, ds);
    return check_launch("softmax_warp_rows_kernel");
}

template <int C, int VPT>
int launch_softmax(float* dst, const float* src, uint64_t rows, uint32_t len, uint64_t ss, uint64_t ds,
                   cudaStream_t stream) {
    const uint64_t blocks = rows * C;
    if (blocks >= (1ull << 31)) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_softmax_lastdim: too many rows");
    if (len == (uint32_t)C * kThreads * 4 * VPT)
        softmax_rows_kernel<C, VPT, true><<<(unsigned)blocks, kThreads, 0, stream>>>(dst, src, len, ss, ds);
    else
        softmax_rows_kernel<C, VPT, false><<<(unsigned)blocks, kThreads, 0, stream>>>(dst, src, len, ss, ds);
    return check_launch("softmax_rows_kernel");
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_softmax_lastdim(int dtype, void* dst, const void* src, uint64_t rows, uint32_t row_len,
                                    uint64_t src_row_stride, uint64_t dst_row_stride) {
    if (int rc = require_init()) return rc;
    if (dtype != MTXC_FLOAT)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_softmax_lastdim: no kernel for dtype ") + dtype_name(dtype));
    if (rows == 0 || row_len == 0) return MTXC_OK;
    if (!dst || !src) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_softmax_lastdim: null buffer");
    if (row_len % 4 || src_row_stride % 4 || dst_row_stride % 4 || !aligned16(dst) || !aligned16(src))
        return fail(MTXC_ERR_INVALID_ARGUMENT,
                    "mtxc_softmax_lastdim: rows must be 16-byte aligned with a length that is a multiple of 4; "
                    "evaluate the unfused trace instead");
    if (row_len > MTXC_SOFTMAX_MAX_ROW)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_softmax_lastdim: row longer than MTXC_SOFTMAX_MAX_ROW; "
                                               "evaluate the unfused trace instead");
    cudaStream_t st = ctx().stream();
    const int sms = ctx().sm_count;
    float* d = static_cast<float*>(dst);
    const float* s = static_cast<const float*>(src);
    const uint32_t vecs = row_len / 4;
    if (vecs <= 32 * 1) return launch_softmax_warps<1>(d, s, rows, row_len, src_row_stride, dst_row_stride, sms, st);
    if (vecs <= 32 * 2) return launch_softmax_warps<2>(d, s, rows, row_len, src_row_stride, dst_row_stride, sms, st);
    if (vecs <= 32 * 4) return launch_softmax_warps<4>(d, s, rows, row_len, src_row_stride, dst_row_stride, sms, st);
    if (vecs <= 32 * 8) return launch_softmax_warps<8>(d, s, rows, row_len, src_row_stride, dst_row_stride, sms, st);
    // 32 elements per thread and the smallest cluster that holds the row: measured on B200 to beat
    // both larger clusters with fewer elements per thread and a cluster-free three-pass kernel
    if (vecs <= 256 * 4) return launch_softmax<1, 4>(d, s, rows, row_len, src_row_stride, dst_row_stride, st);
    if (vecs <= 256 * 8) return launch_softmax<1, 8>(d, s, rows, row_len, src_row_stride, dst_row_stride, st);
    if (vecs <= 512 * 8) return launch_softmax<2, 8>(d, s, rows, row_len, src_row_stride, dst_row_stride, st);
    if (vecs <= 1024 * 8) return launch_softmax<4, 8>(d, s, rows, row_len, src_row_stride, dst_row_stride, st);
    return launch_softmax<8, 8>(d, s, rows, row_len, src_row_stride, dst_row_stride, st);
}
