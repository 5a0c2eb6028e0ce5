// The ordered merge of per-shard partial results for one output, shared by the stand-alone merge kernel
// (merge.cu) and the fused peer-memory exchange (comm.cu).
//
// Part p's value for the output sits at vals[p * vstride] (and its local index at idx[p * istride]).
// Merging in part order keeps the reference's semantics across shards exactly as the kernels keep them
// across CTAs: Sum adds the partials in part order (floats in fp32, rounded once; integers wrap; Bool is a
// logical or); Max / Min take a later part's value only when strictly better, so the first shard wins ties;
// ArgMax / ArgMin do the same on (value, local index) pairs and add the winning part's index offset, so the
// result is the first global index of the extreme -- and 0 when no element beat the initial value, since
// part 0 (offset 0) then wins with its index 0.
#pragma once

#include "mtxc_internal.cuh"

namespace mtxc {

// Writes output gid's merge of `parts` partials to dst[gid] (values; skipped when dst is null) and, for
// ArgMax / ArgMin, dst_idx[gid].
template <int OP, typename T>
__device__ __forceinline__ void merge_one(void* dst, int32_t* dst_idx, const T* vals, uint64_t vstride,
                                          const int32_t* idx, uint64_t istride, uint32_t parts,
                                          const int64_t* offsets, uint64_t gid) {
    if constexpr (OP == MTXC_REDUCE_SUM) {
        if constexpr (Traits<T>::kFloat) {
            float s = to_float(vals[0]);
            for (uint32_t p = 1; p < parts; ++p) s = __fadd_rn(s, to_float(vals[(uint64_t)p * vstride]));
            static_cast<T*>(dst)[gid] = from_float<T>(s);
        } else if constexpr (Traits<T>::kBool) {
            bool s = false;
            for (uint32_t p = 0; p < parts; ++p) s = s || (uint8_t)vals[(uint64_t)p * vstride];
            static_cast<T*>(dst)[gid] = mbool(s);
        } else {
            using W = typename Traits<T>::Acc;
            W s = (W)vals[0];
            for (uint32_t p = 1; p < parts; ++p) s = (W)(s + (W)vals[(uint64_t)p * vstride]);
            static_cast<T*>(dst)[gid] = (T)s;
        }
    } else {
        constexpr bool kMax = (OP == MTXC_REDUCE_MAX || OP == MTXC_REDUCE_ARGMAX);
        T best = vals[0];
        uint32_t from = 0;
        for (uint32_t p = 1; p < parts; ++p) {
            const T x = vals[(uint64_t)p * vstride];
            if (kMax ? less(best, x) : less(x, best)) {
                best = x;
                from = p;
            }
        }
        if (dst) static_cast<T*>(dst)[gid] = best;
        if constexpr (OP == MTXC_REDUCE_ARGMAX || OP == MTXC_REDUCE_ARGMIN)
            dst_idx[gid] = (int32_t)(idx[(uint64_t)from * istride] + offsets[from]);
    }
}

}  // namespace mtxc
