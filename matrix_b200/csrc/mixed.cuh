// Shared by the fused-promotion kernels (mixed.cu: the promoted dtype is one operand's; mixed3.cu: it is
// a third dtype): the element op, which converts each operand to the result dtype as it is read, and the
// dtype code of an element type.
#pragma once

#include "elementwise.cuh"
#include "ops.cuh"
#include "promote.h"

namespace mtxc {

template <typename T>
constexpr int code_of() {
    if constexpr (std::is_same_v<T, float>) return MTXC_FLOAT;
    else if constexpr (std::is_same_v<T, __half>) return MTXC_FLOAT16;
    else if constexpr (std::is_same_v<T, __nv_bfloat16>) return MTXC_BFLOAT16;
    else if constexpr (std::is_same_v<T, int32_t>) return MTXC_INT32;
    else if constexpr (std::is_same_v<T, uint32_t>) return MTXC_UINT32;
    else if constexpr (std::is_same_v<T, int64_t>) return MTXC_INT64;
    else if constexpr (std::is_same_v<T, uint64_t>) return MTXC_UINT64;
    else if constexpr (std::is_same_v<T, int16_t>) return MTXC_INT16;
    else if constexpr (std::is_same_v<T, uint16_t>) return MTXC_UINT16;
    else if constexpr (std::is_same_v<T, int8_t>) return MTXC_INT8;
    else if constexpr (std::is_same_v<T, uint8_t>) return MTXC_UINT8;
    else return MTXC_BOOL;
}

// result D = promote_types(SA, SB); each operand converted to D as it is read, the op in D
template <int OP, typename D, typename SA, typename SB>
struct MixedOp {
    using Out = D;
    using In0 = SA;
    using In1 = SB;
    using In2 = SA;
    static constexpr int kArity = 2;
    __device__ __forceinline__ D operator()(SA a, SB b, SA) const {
        return apply<OP, D>(convert<D, SA>(a), convert<D, SB>(b));
    }
};

// a op b for a pair of operand dtypes that promotes to a third dtype (mixed3.cu); `known` is false when
// no kernel exists for the pair
int launch_mixed3(int op, int dtype, int a_dtype, int b_dtype, const ew::MapDesc& m, int sms, cudaStream_t st,
                  bool& known);

}  // namespace mtxc
