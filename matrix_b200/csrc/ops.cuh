// Element operations shared by the kernels: the reference's binary op on one pair of elements
// (apply) and its dtype_cast conversion (convert).
#pragma once

#include "mtxc_internal.cuh"

namespace mtxc {

// One element of a broadcast binary op (Matrix.mm:7475-7706, 13459-13474, 14757-14781, 14521-14538):
// float-likes compute in fp32 with one rounding (to T for the half types), integers wrap, Bool follows
// C++ bool arithmetic, Max / Min are std::max / std::min selections, Equal writes T(1) or T(0).
template <int OP, typename T>
__device__ __forceinline__ T apply(T x, T y) {
    if constexpr (OP == MTXC_BINARY_EQUAL) {  // matrix::equal: T(1) or T(0) (Matrix.mm:14536)
        if constexpr (Traits<T>::kFloat) return from_float<T>(equal(x, y) ? 1.0f : 0.0f);
        else if constexpr (Traits<T>::kBool) return mbool(x == y);
        else return equal(x, y) ? T(1) : T(0);
    } else if constexpr (OP == MTXC_BINARY_MAX) return less(x, y) ? y : x;  // std::max: x unless x < y
    else if constexpr (OP == MTXC_BINARY_MIN) return less(y, x) ? y : x;  // std::min: x unless y < x
    else if constexpr (Traits<T>::kFloat) {
        // one round-to-nearest operation in fp32; for the half types the fp32 result rounded once to
        // T is the correctly rounded half-precision result (fp32 carries more than 2p + 2 bits)
        const float a = to_float(x), b = to_float(y);
        float r;
        if constexpr (OP == MTXC_BINARY_ADD) r = __fadd_rn(a, b);
        else if constexpr (OP == MTXC_BINARY_SUB) r = __fsub_rn(a, b);
        else if constexpr (OP == MTXC_BINARY_MUL) r = __fmul_rn(a, b);
        else r = __fdiv_rn(a, b);
        return from_float<T>(r);
    } else if constexpr (Traits<T>::kBool) {
        // C++ bool arithmetic: promote to int, convert the result back to bool
        const int a = (uint8_t)x, b = (uint8_t)y;
        int r;
        if constexpr (OP == MTXC_BINARY_ADD) r = a + b;
        else if constexpr (OP == MTXC_BINARY_SUB) r = a - b;
        else if constexpr (OP == MTXC_BINARY_MUL) r = a * b;
        else r = b ? a / b : 0;
        return mbool(r != 0);
    } else {
        // integers: C++ promotion then truncation back to T, with the + - * done in unsigned
        // arithmetic so that overflow wraps as it does on the reference's CPU
        using W = std::conditional_t<(sizeof(T) <= 4), uint32_t, uint64_t>;
        if constexpr (OP == MTXC_BINARY_ADD) return (T)(W)((W)x + (W)y);
        else if constexpr (OP == MTXC_BINARY_SUB) return (T)(W)((W)x - (W)y);
        else if constexpr (OP == MTXC_BINARY_MUL) return (T)(W)((W)x * (W)y);
        else {
            using P = decltype(x / y);  // the promoted type the reference divides in
            return (T)((P)x / (P)y);
        }
    }
}

// apply() over a 16-byte vector of elements.  For the 1-byte types the element-wise ops that need no
// per-byte carries out of a word run on whole 32-bit words: wrapping Add / Sub of int8 / uint8 with the
// per-byte SIMD intrinsics, Bool Add / Sub / Mul as "a or b", "a differs from b", "a and b" per byte
// (C++ bool arithmetic: bool(int(a) + int(b)) ...), each result byte normalised to 0 or 1.  Same results
// as the element loop, a quarter of the instructions.
__device__ __forceinline__ uint32_t nonzero_bytes(uint32_t x) {  // 1 in every byte of x that is not 0
    return ((((x & 0x7f7f7f7fu) + 0x7f7f7f7fu) | x) & 0x80808080u) >> 7;
}

template <int OP, typename T>
__device__ __forceinline__ Vec16<T> apply_vec(const Vec16<T>& x, const Vec16<T>& y) {
    constexpr bool int8_wrap = (std::is_same_v<T, int8_t> || std::is_same_v<T, uint8_t>) &&
                               (OP == MTXC_BINARY_ADD || OP == MTXC_BINARY_SUB);
    constexpr bool bool_logic = std::is_same_v<T, mbool> &&
                                (OP == MTXC_BINARY_ADD || OP == MTXC_BINARY_SUB || OP == MTXC_BINARY_MUL);
    Vec16<T> out;
    if constexpr (int8_wrap || bool_logic) {
        uint32_t a[4], b[4], r[4];
        memcpy(a, &x, 16);
        memcpy(b, &y, 16);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if constexpr (int8_wrap) r[w] = OP == MTXC_BINARY_ADD ? __vadd4(a[w], b[w]) : __vsub4(a[w], b[w]);
            else if constexpr (OP == MTXC_BINARY_ADD) r[w] = nonzero_bytes(a[w] | b[w]);
            else if constexpr (OP == MTXC_BINARY_SUB) r[w] = nonzero_bytes(a[w] ^ b[w]);
            else r[w] = nonzero_bytes(a[w]) & nonzero_bytes(b[w]);
        }
        memcpy(&out, r, 16);
    } else {
#pragma unroll
        for (int j = 0; j < Vec16<T>::N; ++j) out.v[j] = apply<OP, T>(x.v[j], y.v[j]);
    }
    return out;
}

// dtype_cast (matrix.h:260-267) on the device: static_cast, through float between the half types.
//   integer -> integer: the value modulo 2^bits;            integer -> float-like: round to nearest even;
//   float-like -> float-like: round to nearest even;         anything -> bool: x != 0 (NaN is true);
//   bool -> anything: 0 or 1;
//   float-like -> integer: truncation toward zero.  Defined by C++ only when the truncated value fits
//   the destination; outside that range this gives the low bits of the 64-bit truncation (saturated at
//   the int64 range, NaN -> 0).
template <typename T>
constexpr bool kFloatLike = Traits<T>::kFloat;
template <typename T>
constexpr bool kBoolT = std::is_same_v<T, mbool>;

template <typename D, typename S>
__device__ __forceinline__ D convert(S x) {
    if constexpr (std::is_same_v<D, S>) {
        return x;
    } else if constexpr (kBoolT<D>) {
        if constexpr (kFloatLike<S>) return mbool(to_float(x) != 0.0f);
        else return mbool(x != S(0));
    } else if constexpr (kBoolT<S>) {
        const uint32_t v = static_cast<uint8_t>(x) != 0;
        if constexpr (kFloatLike<D>) return from_float<D>((float)v);
        else return D(v);
    } else if constexpr (kFloatLike<D> && kFloatLike<S>) {
        return from_float<D>(to_float(x));  // exact widening, then one rounding
    } else if constexpr (kFloatLike<D>) {  // integer -> float-like
        if constexpr (std::is_same_v<D, float>) {
            return static_cast<float>(x);  // cvt.rn
        } else if constexpr (sizeof(S) <= 2 || std::is_same_v<D, __half>) {
            // exact in float below 2^24; every larger integer rounds to +-inf in half precision
            return from_float<D>(static_cast<float>(x));
        } else if constexpr (std::is_same_v<S, int32_t>) {
            return __int2bfloat16_rn(x);
        } else if constexpr (std::is_same_v<S, uint32_t>) {
            return __uint2bfloat16_rn(x);
        } else if constexpr (std::is_same_v<S, int64_t>) {
            return __ll2bfloat16_rn((long long)x);
        } else {
            return __ull2bfloat16_rn((unsigned long long)x);
        }
    } else if constexpr (kFloatLike<S>) {  // float-like -> integer
        const float f = to_float(x);
        if constexpr (std::is_same_v<D, uint64_t>) {
            if (f >= 9223372036854775808.0f) return (uint64_t)__float2ull_rz(f);
        }
        return static_cast<D>((uint64_t)__float2ll_rz(f));
    } else {
        return static_cast<D>(x);  // integer -> integer: modulo 2^bits
    }
}

}  // namespace mtxc
