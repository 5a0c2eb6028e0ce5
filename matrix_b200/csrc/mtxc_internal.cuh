// Internal definitions shared by the mtxc translation units: the per-thread runtime context,
// error reporting, dtype dispatch, 32-bit fast division and the 128-bit memory helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <string>
#include <type_traits>

#include "mtxc.h"

namespace mtxc {

struct CommState;  // comm.cu: the thread's multi-GPU communicator

// ------------------------------------------------------------------------------------------
// Runtime context: one per host thread, the analogue of the reference's thread-local command
// buffer and encoder (Mods/GPUManager.h:57-58).
// ------------------------------------------------------------------------------------------
struct ThreadCtx {
    int device = -1;
    cudaStream_t own_stream = nullptr;   // created by mtxc_init
    cudaStream_t user_stream = nullptr;  // set by mtxc_set_stream (may be the default stream, 0)
    bool has_user_stream = false;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    bool own_workspace = false;
    int sm_count = 148;
    CommState* comm = nullptr;           // set by mtxc_comm_init
    std::string last_error;
    cudaStream_t stream() const { return has_user_stream ? user_stream : own_stream; }
};

ThreadCtx& ctx();
// Destroys the calling thread's communicator, if any (comm.cu).
void comm_release();
// Drops mtxc_reduce_noalloc's cached scratch address for a device (reduce.cu).
void noalloc_forget(int device);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t err, const char* what);
// Checks that mtxc_init ran on this thread; returns MTXC_OK or an error status.
int require_init();
// Checks the launch that just happened; returns MTXC_OK or MTXC_ERR_CUDA.
int check_launch(const char* what);

// ------------------------------------------------------------------------------------------
// Element types.  The reference's Bool (dtype 7) is a 1-byte 0/1 value with C++ bool semantics: a
// scoped enum over uint8 keeps it distinct from UInt8 in every template below.
// ------------------------------------------------------------------------------------------
enum class mbool : uint8_t {};

template <typename T>
struct Traits {  // integers
    static constexpr bool kFloat = false, kBool = false;
    using Acc = std::conditional_t<(sizeof(T) <= 4), uint32_t, uint64_t>;  // wrap-around accumulator
};
template <>
struct Traits<float> {
    static constexpr bool kFloat = true, kBool = false;
    using Acc = float;
};
template <>
struct Traits<__half> {
    static constexpr bool kFloat = true, kBool = false;
    using Acc = float;
};
template <>
struct Traits<__nv_bfloat16> {
    static constexpr bool kFloat = true, kBool = false;
    using Acc = float;
};
template <>
struct Traits<mbool> {
    static constexpr bool kFloat = false, kBool = true;
    using Acc = uint32_t;
};

// Exact widening of a float-like element to float (identity for float).
template <typename T>
__host__ __device__ __forceinline__ float to_float(T v) {
    if constexpr (std::is_same_v<T, float>) return v;
    else if constexpr (std::is_same_v<T, __half>) return __half2float(v);
    else return __bfloat162float(v);
}
// Round-to-nearest-even narrowing of a float to a float-like element.
template <typename T>
__host__ __device__ __forceinline__ T from_float(float v) {
    if constexpr (std::is_same_v<T, float>) return v;
    else if constexpr (std::is_same_v<T, __half>) return __float2half_rn(v);
    else return __float2bfloat16_rn(v);
}
// a < b in the element's own order (float-likes compare as floats: exact, NaN is unordered).
template <typename T>
__host__ __device__ __forceinline__ bool less(T a, T b) {
    if constexpr (Traits<T>::kFloat) return to_float(a) < to_float(b);
    else return a < b;
}
template <typename T>
__host__ __device__ __forceinline__ bool equal(T a, T b) {
    if constexpr (Traits<T>::kFloat) return to_float(a) == to_float(b);
    else return a == b;
}

template <typename Fn>
bool dispatch_dtype(int dtype, Fn&& fn) {
    switch (dtype) {
        case MTXC_FLOAT: fn((float*)nullptr); return true;
        case MTXC_FLOAT16: fn((__half*)nullptr); return true;
        case MTXC_BFLOAT16: fn((__nv_bfloat16*)nullptr); return true;
        case MTXC_INT32: fn((int32_t*)nullptr); return true;
        case MTXC_UINT32: fn((uint32_t*)nullptr); return true;
        case MTXC_INT64: fn((int64_t*)nullptr); return true;
        case MTXC_UINT64: fn((uint64_t*)nullptr); return true;
        case MTXC_INT16: fn((int16_t*)nullptr); return true;
        case MTXC_UINT16: fn((uint16_t*)nullptr); return true;
        case MTXC_INT8: fn((int8_t*)nullptr); return true;
        case MTXC_UINT8: fn((uint8_t*)nullptr); return true;
        case MTXC_BOOL: fn((mbool*)nullptr); return true;
        default: return false;
    }
}
const char* dtype_name(int dtype);

// Smallest / largest finite value: dtype_lowest / dtype_max (matrix.h:271-282), with the half types'
// finite extremes (+-65504, +-0x1.fep127) and bool's false / true.
template <typename T>
__host__ __device__ inline T lowest_value() {
    if constexpr (std::is_same_v<T, float>) return -3.402823466e+38f;
    else if constexpr (std::is_same_v<T, __half>) return __ushort_as_half((unsigned short)0xFBFFu);
    else if constexpr (std::is_same_v<T, __nv_bfloat16>) return __ushort_as_bfloat16((unsigned short)0xFF7Fu);
    else if constexpr (std::is_same_v<T, mbool>) return mbool(0);
    else if constexpr (std::is_signed_v<T>) return T(T(1) << (sizeof(T) * 8 - 1));
    else return T(0);
}
template <typename T>
__host__ __device__ inline T highest_value() {
    if constexpr (std::is_same_v<T, float>) return 3.402823466e+38f;
    else if constexpr (std::is_same_v<T, __half>) return __ushort_as_half((unsigned short)0x7BFFu);
    else if constexpr (std::is_same_v<T, __nv_bfloat16>) return __ushort_as_bfloat16((unsigned short)0x7F7Fu);
    else if constexpr (std::is_same_v<T, mbool>) return mbool(1);
    else if constexpr (std::is_signed_v<T>) return T(~(T(1) << (sizeof(T) * 8 - 1)));
    else return T(~T(0));
}

// ------------------------------------------------------------------------------------------
// Metadata passed by value to kernels.
// ------------------------------------------------------------------------------------------
// Division by a runtime-invariant 32-bit divisor via a multiply-high (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994, round-up variant):
// q = (umulhi(n, m) + n) >> s with s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1.
// Exact for every 32-bit n and 1 <= d < 2^31.
struct FastDiv {
    uint32_t d = 1, m = 0, s = 0;
    FastDiv() = default;
    explicit FastDiv(uint32_t div) : d(div) {
        s = 0;
        while ((1ull << s) < div) ++s;
        m = (uint32_t)(((1ull << 32) * ((1ull << s) - div)) / div + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return (uint32_t)(((uint64_t)__umulhi(n, m) + n) >> s);
    }
    __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
        q = div(n);
        r = n - q * d;
    }
};

// Per-axis metadata (reference collapsed dims), at most MTXC_MAX_DIMS axes.
struct Dims {
    uint32_t n = 0;
    uint32_t shape[MTXC_MAX_DIMS];
    uint32_t s0[MTXC_MAX_DIMS];
    uint32_t s1[MTXC_MAX_DIMS];
    uint32_t s2[MTXC_MAX_DIMS];
    FastDiv fdiv[MTXC_MAX_DIMS];  // per-axis divisor (shape or stride, as the kernel needs)
};

inline uint64_t product(const uint32_t* shape, uint32_t n) {
    uint64_t p = 1;
    for (uint32_t i = 0; i < n; ++i) p *= shape[i];
    return p;
}

// True when strides are the row-major strides of shape (axes of extent 1 are ignored).
inline bool is_row_major(const uint32_t* shape, const uint32_t* strides, uint32_t n) {
    uint64_t acc = 1;
    for (int i = (int)n - 1; i >= 0; --i) {
        if (shape[i] != 1 && strides[i] != acc) return false;
        acc *= shape[i];
    }
    return true;
}

// ------------------------------------------------------------------------------------------
// 128-bit memory helpers.
// ------------------------------------------------------------------------------------------
template <typename T>
struct alignas(16) Vec16 {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

// Streaming read that bypasses L1 (data read once).  Not volatile: the compiler may schedule it
// freely, e.g. hoist several loads ahead of their first use.  Every kernel here reads an element
// before anything writes it (in-place exp writes an element only with a value computed from its own
// load), so no ordering against stores is needed.
template <typename T>
__device__ __forceinline__ Vec16<T> load_stream(const T* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    Vec16<T> out;
    memcpy(&out, &r, 16);
    return out;
}
// Read through the read-only path (data reused across threads: broadcast operands).
template <typename T>
__device__ __forceinline__ Vec16<T> load_cached(const T* p) {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    Vec16<T> out;
    memcpy(&out, &r, 16);
    return out;
}
// Streaming scalar read of any 1/2/4/8-byte element type.
template <typename T>
__device__ __forceinline__ T load_scalar_stream(const T* p) {
    T out;
    if constexpr (sizeof(T) == 8) {
        unsigned long long r = __ldcs(reinterpret_cast<const unsigned long long*>(p));
        memcpy(&out, &r, 8);
    } else if constexpr (sizeof(T) == 4) {
        unsigned int r = __ldcs(reinterpret_cast<const unsigned int*>(p));
        memcpy(&out, &r, 4);
    } else if constexpr (sizeof(T) == 2) {
        unsigned short r = __ldcs(reinterpret_cast<const unsigned short*>(p));
        memcpy(&out, &r, 2);
    } else {
        unsigned char r = __ldcs(reinterpret_cast<const unsigned char*>(p));
        memcpy(&out, &r, 1);
    }
    return out;
}
// Streaming (evict-first) store: the output is written once and not re-read by this op.
template <typename T>
__device__ __forceinline__ void store_stream(T* p, const Vec16<T>& v) {
    uint4 r;
    memcpy(&r, &v, 16);
    __stcs(reinterpret_cast<uint4*>(p), r);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace mtxc
