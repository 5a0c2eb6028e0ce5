// Ordered merge of per-shard partial reductions: the cross-GPU step of a reduction whose reduced
// axis is sharded across GPUs (benchmark configs 4 and 5b).
//
// Each of `parts` shards reduced its contiguous slice of the axis; their partial results arrive
// part-major (part p's `outputs` results at p * outputs, in shard order, e.g. from an NCCL
// all-gather) and are merged in part order (merge_one, merge.cuh).
#include <algorithm>

#include "merge.cuh"

namespace mtxc {
namespace {

constexpr int kBlock = 256;
constexpr uint32_t kMaxParts = 256;

struct MergeArgs {
    void* dst;
    int32_t* dst_idx;
    const void* vals;
    const int32_t* idx;
    uint64_t outputs;
    uint32_t parts;
    int64_t offsets[kMaxParts];
};

template <int OP, typename T>
__global__ void __launch_bounds__(kBlock) merge_partials_kernel(const MergeArgs a) {
    const T* v = static_cast<const T*>(a.vals);
    for (uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < a.outputs;
         gid += (uint64_t)gridDim.x * blockDim.x)
        merge_one<OP, T>(a.dst, a.dst_idx, v + gid, a.outputs, a.idx ? a.idx + gid : nullptr, a.outputs, a.parts,
                         a.offsets, gid);
}

template <typename T>
int launch_merge(int op, const MergeArgs& a, int sm_count, cudaStream_t st) {
    const uint64_t blocks = std::max<uint64_t>(1, std::min<uint64_t>((a.outputs + kBlock - 1) / kBlock, (uint64_t)sm_count * 8));
    switch (op) {
        case MTXC_REDUCE_SUM: merge_partials_kernel<MTXC_REDUCE_SUM, T><<<(unsigned)blocks, kBlock, 0, st>>>(a); break;
        case MTXC_REDUCE_MAX: merge_partials_kernel<MTXC_REDUCE_MAX, T><<<(unsigned)blocks, kBlock, 0, st>>>(a); break;
        case MTXC_REDUCE_MIN: merge_partials_kernel<MTXC_REDUCE_MIN, T><<<(unsigned)blocks, kBlock, 0, st>>>(a); break;
        case MTXC_REDUCE_ARGMAX: merge_partials_kernel<MTXC_REDUCE_ARGMAX, T><<<(unsigned)blocks, kBlock, 0, st>>>(a); break;
        default: merge_partials_kernel<MTXC_REDUCE_ARGMIN, T><<<(unsigned)blocks, kBlock, 0, st>>>(a); break;
    }
    return check_launch("merge_partials_kernel");
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_merge_partials(int op, int dtype, void* dst, int32_t* dst_indices, const void* part_values,
                                   const int32_t* part_indices, const int64_t* index_offsets, uint32_t parts,
                                   uint64_t outputs) {
    if (int rc = require_init()) return rc;
    if (op < MTXC_REDUCE_SUM || op > MTXC_REDUCE_ARGMIN)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_merge_partials: unknown op");
    if (parts == 0 || parts > kMaxParts)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_merge_partials: parts must be in [1, 256]");
    if (outputs == 0) return MTXC_OK;
    const bool arg = op == MTXC_REDUCE_ARGMAX || op == MTXC_REDUCE_ARGMIN;
    if (!part_values || (arg && (!dst_indices || !part_indices || !index_offsets)) || (!arg && !dst))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_merge_partials: null buffer");
    MergeArgs a{};
    a.dst = dst;
    a.dst_idx = dst_indices;
    a.vals = part_values;
    a.idx = part_indices;
    a.outputs = outputs;
    a.parts = parts;
    for (uint32_t p = 0; p < parts && arg; ++p) a.offsets[p] = index_offsets[p];
    ThreadCtx& c = ctx();
    int rc = MTXC_OK;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_merge<T>(op, a, c.sm_count, c.stream());
    });
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_merge_partials: no kernel for dtype ") + dtype_name(dtype));
    return rc;
}
