// CPU oracle for the reduce / broadcast hot path of AlanAditya/matrix.
//
// TEST INFRASTRUCTURE ONLY.  This file restates, loop for loop, the reference's
// own CPU evaluation of the hot-path primitives so that the CUDA backend can be
// checked against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline leg load it; the product library (matrix_b200/) never does.
//
// Every function names the reference lines it restates (paths are relative to
// the reference project root).  What is kept on purpose:
//   * loop order, initial values and accumulator type T (sequential fp32 sums,
//     wrap-around integer sums, std::max / std::min selection semantics,
//     strict > / < for ArgMax / ArgMin so the first index wins);
//   * the stride-division index decode of the reduction and broadcast loops;
//   * uint32 (size_m) arithmetic inside the shape-folding helpers.
// What differs: loop indices are 64-bit (the reference's `int gid` / size_m
// counters would overflow past 2^31 elements), and the output range can be
// split across host threads.  Every thread runs the identical scalar loop on
// its own slice of outputs, so results do not depend on the thread count.
//
// Parity pin: oracle/build_ref.py compiles the reference's own CPU loops and
// shape-folding functions, taken from where they lie in the reference tree,
// into oracle/_ref/libmtx_ref.so; tests/test_oracle_pin.py compares the two on
// random cases, and tests/golden/ holds fixtures generated from that library.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <type_traits>
#include <vector>

namespace {

using size_m = uint32_t;  // Mods/Utils.h:125
constexpr uint32_t kMaxDims = 8;  // MAX_TENSOR_DIMS, Mods/Utils.h:127

// dtype codes, matrix.h:35-51
enum Dtype : int {
    kFloat = 0, kFloat16 = 1, kUInt8 = 2, kInt32 = 3, kInt16 = 4, kUInt32 = 5,
    kUInt16 = 6, kBool = 7, kInt8 = 8, kComplex64 = 9, kBFloat16 = 10,
    kInt64 = 11, kUInt64 = 12
};

// dtype_lowest / dtype_max, matrix.h:271-282: numeric_limits except for the
// two half types, whose finite extremes are spelled out.
template <typename T> inline T lowest_of() {
    if constexpr (std::is_same_v<T, _Float16>) return static_cast<T>(-65504.0f);
    else if constexpr (std::is_same_v<T, __bf16>) return static_cast<T>(-0x1.fep127f);
    else return std::numeric_limits<T>::lowest();
}
template <typename T> inline T highest_of() {
    if constexpr (std::is_same_v<T, _Float16>) return static_cast<T>(65504.0f);
    else if constexpr (std::is_same_v<T, __bf16>) return static_cast<T>(0x1.fep127f);
    else return std::numeric_limits<T>::max();
}

// Runs fn(T*) for the element type of `code`; returns false for Complex64,
// mirroring dispatch_type's refusal of it (matrix.h:284-334).  Bool runs with
// C++ bool arithmetic: the int result of `a + b` etc. converted back to bool.
template <typename Fn> bool with_type(int code, Fn&& fn) {
    switch (code) {
        case kFloat: fn((float*)nullptr); return true;
        case kFloat16: fn((_Float16*)nullptr); return true;
        case kUInt8: fn((uint8_t*)nullptr); return true;
        case kInt32: fn((int32_t*)nullptr); return true;
        case kInt16: fn((int16_t*)nullptr); return true;
        case kUInt32: fn((uint32_t*)nullptr); return true;
        case kUInt16: fn((uint16_t*)nullptr); return true;
        case kInt8: fn((int8_t*)nullptr); return true;
        case kBool: fn((bool*)nullptr); return true;
        case kBFloat16: fn((__bf16*)nullptr); return true;
        case kInt64: fn((int64_t*)nullptr); return true;
        case kUInt64: fn((uint64_t*)nullptr); return true;
        default: return false;
    }
}

// Integer addition in the reference wraps (two's complement); do it in the
// unsigned type of the same width so the restatement has no signed overflow.
template <typename T> inline T add_wrap(T a, T b) {
    if constexpr (std::is_same_v<T, bool>) {
        return static_cast<bool>(int(a) + int(b));
    } else if constexpr (std::is_integral_v<T>) {
        using U = std::make_unsigned_t<T>;
        return static_cast<T>(static_cast<U>(static_cast<U>(a) + static_cast<U>(b)));
    } else {
        return static_cast<T>(a + b);
    }
}
template <typename T> inline T sub_wrap(T a, T b) {
    if constexpr (std::is_same_v<T, bool>) {
        return static_cast<bool>(int(a) - int(b));
    } else if constexpr (std::is_integral_v<T>) {
        using U = std::make_unsigned_t<T>;
        return static_cast<T>(static_cast<U>(static_cast<U>(a) - static_cast<U>(b)));
    } else {
        return static_cast<T>(a - b);
    }
}
template <typename T> inline T mul_wrap(T a, T b) {
    if constexpr (std::is_same_v<T, bool>) {
        return static_cast<bool>(int(a) * int(b));
    } else if constexpr (std::is_integral_v<T>) {
        using U = std::make_unsigned_t<T>;
        // promote narrow unsigned types to unsigned int before multiplying so
        // the product itself cannot overflow a signed int
        using W = std::conditional_t<(sizeof(U) < sizeof(unsigned)), unsigned, U>;
        return static_cast<T>(static_cast<W>(static_cast<W>(static_cast<U>(a)) * static_cast<W>(static_cast<U>(b))));
    } else {
        return static_cast<T>(a * b);
    }
}

template <typename T> constexpr bool kFloatLike =
    std::is_same_v<T, float> || std::is_same_v<T, _Float16> || std::is_same_v<T, __bf16>;

// dtype_cast, matrix.h:260-267: a static_cast, through float between the two half types.  A
// float-like value converted to an integer type is defined in C++ only when its truncation fits the
// destination; the restatement gives such values the low bits of the 64-bit truncation (saturated at
// the int64 range, NaN -> 0) instead of undefined behaviour, and the tests compare in-range values.
template <typename D, typename S> inline D cast_elem(S v) {
    if constexpr (std::is_same_v<D, S>) {
        return v;
    } else if constexpr (std::is_same_v<D, bool>) {
        return static_cast<bool>(v);
    } else if constexpr (kFloatLike<S> && std::is_integral_v<D>) {
        const float f = static_cast<float>(v);
        if constexpr (std::is_same_v<D, uint64_t>) {
            if (f >= 0x1p63f) return f >= 0x1p64f ? UINT64_MAX : static_cast<uint64_t>(f);
        }
        int64_t t;
        if (std::isnan(f)) t = 0;
        else if (f >= 0x1p63f) t = INT64_MAX;
        else if (f < -0x1p63f) t = INT64_MIN;
        else t = static_cast<int64_t>(f);
        return static_cast<D>(static_cast<uint64_t>(t));
    } else if constexpr ((std::is_same_v<S, _Float16> && std::is_same_v<D, __bf16>) ||
                         (std::is_same_v<S, __bf16> && std::is_same_v<D, _Float16>)) {
        return static_cast<D>(static_cast<float>(v));
    } else {
        return static_cast<D>(v);
    }
}

// Splits [0, n) into `threads` contiguous slices and runs body(lo, hi) on each.
template <typename Body> void parallel_ranges(uint64_t n, int threads, Body&& body) {
    if (threads <= 1 || n < 4096) { body(uint64_t(0), n); return; }
    uint64_t t = std::min<uint64_t>(threads, n);
    std::vector<std::thread> pool;
    pool.reserve(t);
    for (uint64_t k = 0; k < t; ++k) {
        uint64_t lo = n * k / t, hi = n * (k + 1) / t;
        pool.emplace_back([&body, lo, hi] { body(lo, hi); });
    }
    for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Shape folding.  All arithmetic is in uint32 (size_m) exactly as in the
// reference, including the product compared against SIZE_CAP.
// ---------------------------------------------------------------------------

// collapse_dims, one operand: Mods/Utils.mm:114-136
uint32_t orc_collapse1(const uint32_t* shape, const uint32_t* s0, uint32_t dims, uint64_t cap,
                       uint32_t* oshape, uint32_t* os0) {
    if (dims == 0) return 0;
    oshape[0] = shape[0];
    os0[0] = s0[0];
    uint32_t last = 0;
    for (uint32_t i = 1; i < dims; ++i) {
        if (shape[i] == 1) continue;
        const size_m prod = oshape[last] * shape[i];
        if (os0[last] != s0[i] * shape[i] || prod > cap) {
            ++last;
            oshape[last] = shape[i];
            os0[last] = s0[i];
        } else {
            oshape[last] = prod;
            os0[last] = s0[i];
        }
    }
    return last + 1;
}

// collapse_dims, two operands: Mods/Utils.mm:138-166
uint32_t orc_collapse2(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, uint32_t dims,
                       uint64_t cap, uint32_t* oshape, uint32_t* os0, uint32_t* os1) {
    if (dims == 0) return 0;
    oshape[0] = shape[0];
    os0[0] = s0[0];
    os1[0] = s1[0];
    uint32_t last = 0;
    for (uint32_t i = 1; i < dims; ++i) {
        if (shape[i] == 1) continue;
        const size_m prod = oshape[last] * shape[i];
        const bool contiguous = os0[last] == s0[i] * shape[i] && os1[last] == s1[i] * shape[i];
        if (!contiguous || prod > cap) {
            ++last;
            oshape[last] = shape[i];
        } else {
            oshape[last] = prod;
        }
        os0[last] = s0[i];
        os1[last] = s1[i];
    }
    return last + 1;
}

// collapse_dims, three operands: Mods/Utils.mm:169-202
uint32_t orc_collapse3(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, const uint32_t* s2,
                       uint32_t dims, uint64_t cap, uint32_t* oshape, uint32_t* os0, uint32_t* os1,
                       uint32_t* os2) {
    if (dims == 0) return 0;
    oshape[0] = shape[0];
    os0[0] = s0[0];
    os1[0] = s1[0];
    os2[0] = s2[0];
    uint32_t last = 0;
    for (uint32_t i = 1; i < dims; ++i) {
        if (shape[i] == 1) continue;
        const size_m prod = oshape[last] * shape[i];
        const bool contiguous = os0[last] == s0[i] * shape[i] && os1[last] == s1[i] * shape[i] &&
                                os2[last] == s2[i] * shape[i];
        if (!contiguous || prod > cap) {
            ++last;
            oshape[last] = shape[i];
        } else {
            oshape[last] = prod;
        }
        os0[last] = s0[i];
        os1[last] = s1[i];
        os2[last] = s2[i];
    }
    return last + 1;
}

// collapse_dims_reduce, one operand: Mods/Utils.mm:270-319
uint32_t orc_collapse_reduce1(const uint32_t* shape, const uint32_t* so, uint32_t dims, int axis,
                              int keep_dims, uint64_t cap, uint32_t* oshape, uint32_t* oso) {
    if (dims == 0) return 0;
    int last = -1;
    bool split = false;
    for (int i = 0; i < (int)dims; ++i) {
        if (i == axis) {
            if (keep_dims) {
                ++last;
                oshape[last] = shape[i];
                oso[last] = so[i];
            }
            split = true;
            continue;
        }
        if (shape[i] == 1) continue;
        if (!split && last >= 0 && oso[last] == so[i] * shape[i] && (size_m)(oshape[last] * shape[i]) <= cap) {
            oshape[last] *= shape[i];
            oso[last] = so[i];
        } else {
            ++last;
            oshape[last] = shape[i];
            oso[last] = so[i];
            split = false;
        }
    }
    return (uint32_t)(last + 1);
}

// collapse_dims_reduce, two operands (output strides, input strides):
// Mods/Utils.mm:321-376.  With outer_collapsed the output has one axis fewer
// than the input, so output strides past the reduced axis are read one slot
// to the left.
uint32_t orc_collapse_reduce2(const uint32_t* shape, const uint32_t* so, const uint32_t* si, uint32_t dims,
                              int axis, int keep_dims, int outer_collapsed, uint64_t cap, uint32_t* oshape,
                              uint32_t* oso, uint32_t* osi) {
    if (dims == 0) return 0;
    int last = -1;
    bool split = false;
    for (int i = 0; i < (int)dims; ++i) {
        if (i == axis) {
            if (keep_dims) {
                ++last;
                oshape[last] = shape[i];
                oso[last] = so[i];
                osi[last] = si[i];
            }
            split = true;
            continue;
        }
        if (shape[i] == 1) continue;
        const int oi = (outer_collapsed && axis < i) ? i - 1 : i;
        if (!split && last >= 0 && oso[last] == so[oi] * shape[i] && osi[last] == si[i] * shape[i] &&
            (size_m)(oshape[last] * shape[i]) <= cap) {
            oshape[last] *= shape[i];
            oso[last] = so[oi];
            osi[last] = si[i];
        } else {
            ++last;
            oshape[last] = shape[i];
            oso[last] = so[oi];
            osi[last] = si[i];
            split = false;
        }
    }
    return (uint32_t)(last + 1);
}

// collapse_dims_reduce, three operands: Mods/Utils.mm:378-435
uint32_t orc_collapse_reduce3(const uint32_t* shape, const uint32_t* so, const uint32_t* sb, const uint32_t* sc,
                              uint32_t dims, int axis, int keep_dims, uint64_t cap, uint32_t* oshape,
                              uint32_t* oso, uint32_t* osb, uint32_t* osc) {
    if (dims == 0) return 0;
    int last = -1;
    bool split = false;
    for (int i = 0; i < (int)dims; ++i) {
        if (i == axis) {
            if (keep_dims) {
                ++last;
                oshape[last] = shape[i];
                oso[last] = so[i];
                osb[last] = sb[i];
                osc[last] = sc[i];
            }
            split = true;
            continue;
        }
        if (shape[i] == 1) continue;
        if (!split && last >= 0 && oso[last] == so[i] * shape[i] && osb[last] == sb[i] * shape[i] &&
            osc[last] == sc[i] * shape[i] && (size_m)(oshape[last] * shape[i]) <= cap) {
            oshape[last] *= shape[i];
            oso[last] = so[i];
            osb[last] = sb[i];
            osc[last] = sc[i];
        } else {
            ++last;
            oshape[last] = shape[i];
            oso[last] = so[i];
            osb[last] = sb[i];
            osc[last] = sc[i];
            split = false;
        }
    }
    return (uint32_t)(last + 1);
}

// broadcast_shapes: Matrix.mm:161-232.  Right-aligned NumPy broadcasting; an
// operand axis of extent 1 that meets a larger extent gets stride 0; leading
// axes an operand lacks get stride 0.  Returns 0, or -1 where the reference
// throws std::invalid_argument (Matrix.mm:220).
int orc_broadcast_shapes(const uint32_t* shape1, const uint32_t* strides1, int dim1, const uint32_t* shape2,
                         const uint32_t* strides2, int dim2, uint32_t* out_shape, uint32_t* out_strides,
                         uint32_t* a_shape, uint32_t* a_strides, uint32_t* b_shape, uint32_t* b_strides) {
    const int od = std::max(dim1, dim2);
    for (int i = 0; i < od; ++i) {
        a_strides[i] = 0;
        b_strides[i] = 0;
        a_shape[i] = 0;
        b_shape[i] = 0;
    }
    for (int i = 0; i < dim1; ++i) {
        a_strides[od - dim1 + i] = strides1[i];
        a_shape[od - dim1 + i] = shape1[i];
    }
    for (int i = 0; i < dim2; ++i) {
        b_strides[od - dim2 + i] = strides2[i];
        b_shape[od - dim2 + i] = shape2[i];
    }
    for (int i = 0; i < od; ++i) {
        const int o = od - i - 1;
        if (dim1 < i + 1) {
            a_shape[o] = shape2[dim2 - i - 1];
            out_shape[o] = shape2[dim2 - i - 1];
        } else if (dim2 < i + 1) {
            b_shape[o] = shape1[dim1 - i - 1];
            out_shape[o] = shape1[dim1 - i - 1];
        } else {
            const uint32_t e1 = shape1[dim1 - i - 1], e2 = shape2[dim2 - i - 1];
            if (e1 == e2) {
                out_shape[o] = e1;
            } else if (e1 == 1) {
                a_shape[o] = e2;
                out_shape[o] = e2;
                a_strides[o] = 0;
            } else if (e2 == 1) {
                b_shape[o] = e1;
                out_shape[o] = e1;
                b_strides[o] = 0;
            } else {
                return -1;
            }
        }
    }
    size_m acc = 1;
    for (int i = od - 1; i >= 0; --i) {
        out_strides[i] = acc;
        acc *= out_shape[i];
    }
    return 0;
}

// promote_types: Matrix.mm:107-109 over the table at matrix.h:166-180.
int orc_promote(int a, int b) {
    // rows/columns in dtype-code order: F F16 U8 I32 I16 U32 U16 B I8 C64 BF16 I64 U64
    static const signed char rules[13][13] = {
        {0, 0, 0, 0, 0, 0, 0, 0, 0, 9, 0, 0, 0},
        {0, 1, 0, 0, 0, 0, 0, 1, 0, 9, 0, 0, 0},
        {0, 0, 2, 3, 4, 5, 6, 2, 4, 9, 0, 11, 12},
        {0, 0, 3, 3, 3, 3, 3, 3, 3, 9, 0, 11, 0},
        {0, 0, 4, 3, 4, 3, 3, 4, 4, 9, 0, 11, 0},
        {0, 0, 5, 3, 3, 5, 5, 5, 3, 9, 0, 11, 12},
        {0, 0, 6, 3, 3, 5, 6, 6, 3, 9, 0, 11, 12},
        {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12},
        {0, 0, 4, 3, 4, 3, 3, 8, 8, 9, 0, 11, 0},
        {9, 9, 9, 9, 9, 9, 9, 9, 9, 9, 9, 9, 9},
        {0, 0, 0, 0, 0, 0, 0, 10, 0, 9, 10, 0, 0},
        {0, 0, 11, 11, 11, 11, 11, 11, 11, 9, 0, 11, 0},
        {0, 0, 12, 0, 0, 12, 12, 12, 0, 9, 0, 0, 12},
    };
    if (a < 0 || a > 12 || b < 0 || b > 12) return -1;
    return rules[a][b];
}

// ---------------------------------------------------------------------------
// Full Sum of a contiguous tensor: matrix::sum() (Matrix.mm:15215-15218) is flatten(0, -1).sum(0), one
// output whose run is every element in memory order, summed by the Sum loop (Matrix.mm:15201-15204:
// acc = 0; acc += x, in T).  The count is 64-bit because benchmark config 5b's 2^32 elements do not fit
// the reference's 32-bit size_m (its flatten would wrap the extent to 0); the loop is otherwise the
// reference's, sequential on one thread.
// ---------------------------------------------------------------------------
int orc_sum_flat(int dtype, void* out, const void* in, uint64_t n) {
    const bool ok = with_type(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        const T* p = static_cast<const T*>(in);
        T acc = static_cast<T>(0);
        for (uint64_t i = 0; i < n; ++i) acc = add_wrap<T>(acc, p[i]);
        *static_cast<T*>(out) = acc;
    });
    return ok ? 0 : -1;
}

// ---------------------------------------------------------------------------
// Axis reductions.  op: 0 Sum, 1 Max, 2 Min, 3 ArgMax, 4 ArgMin.
//   Sum    Matrix.mm:15187-15207   acc = 0; acc += x            (T accumulator)
//   Max    Matrix.mm:14894-14914   acc = lowest; std::max(acc, x)
//   Min    Matrix.mm:15038-15058   acc = max;    std::min(acc, x)
//   ArgMax Matrix.mm:16279-16302   (lowest, 0); take x when x > best
//   ArgMin Matrix.mm:16434-16457   (max, 0);    take x when x < best
// Output element gid is written at out[gid]; its input offset comes from
// dividing gid by the collapsed output strides sA and scaling by the input
// strides sB.  cdims == 0 means one output at offset 0 (Matrix.mm:15121-15126).
// ArgMax / ArgMin write int32.  Returns 0, or -1 for an unsupported dtype / op.
// ---------------------------------------------------------------------------
int orc_reduce(int op, int dtype, void* out, const void* in, uint32_t rstride, uint32_t rlen, uint32_t cdims,
               const uint32_t* shape_unused, const uint32_t* sA_in, const uint32_t* sB_in, uint64_t total_out,
               int threads) {
    (void)shape_unused;
    uint32_t sA[kMaxDims], sB[kMaxDims];
    if (cdims > kMaxDims || op < 0 || op > 4) return -1;
    if (cdims == 0) {
        cdims = 1;
        sA[0] = 1;
        sB[0] = 1;
    } else {
        for (uint32_t i = 0; i < cdims; ++i) {
            sA[i] = sA_in[i];
            sB[i] = sB_in[i];
        }
    }
    int status = 0;
    const bool ok = with_type(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        const T* src = static_cast<const T*>(in);
        parallel_ranges(total_out, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t gid = lo; gid < hi; ++gid) {
                uint64_t off = 0, rem = gid;
                for (uint32_t i = 0; i < cdims; ++i) {
                    off += (rem / sA[i]) * sB[i];
                    rem %= sA[i];
                }
                const T* p = src + off;
                if (op == 0) {
                    T acc = static_cast<T>(0);
                    for (uint64_t i = 0; i < rlen; ++i) acc = add_wrap<T>(acc, p[i * rstride]);
                    static_cast<T*>(out)[gid] = acc;
                } else if (op == 1) {
                    T acc = lowest_of<T>();
                    for (uint64_t i = 0; i < rlen; ++i) acc = std::max(acc, p[i * rstride]);
                    static_cast<T*>(out)[gid] = acc;
                } else if (op == 2) {
                    T acc = highest_of<T>();
                    for (uint64_t i = 0; i < rlen; ++i) acc = std::min(acc, p[i * rstride]);
                    static_cast<T*>(out)[gid] = acc;
                } else if (op == 3) {
                    T best = lowest_of<T>();
                    int32_t arg = 0;
                    for (uint64_t i = 0; i < rlen; ++i) {
                        const T v = p[i * rstride];
                        if (v > best) {
                            best = v;
                            arg = (int32_t)i;
                        }
                    }
                    static_cast<int32_t*>(out)[gid] = arg;
                } else {
                    T best = highest_of<T>();
                    int32_t arg = 0;
                    for (uint64_t i = 0; i < rlen; ++i) {
                        const T v = p[i * rstride];
                        if (v < best) {
                            best = v;
                            arg = (int32_t)i;
                        }
                    }
                    static_cast<int32_t*>(out)[gid] = arg;
                }
            }
        });
    });
    if (!ok) status = -1;
    return status;
}

// ---------------------------------------------------------------------------
// Broadcast binary ops.  op: 0 Add, 1 Sub, 2 Mul, 3 Div, 4 Max, 5 Min, 6 Equal.
//   add/mul/sub/div  Matrix.mm:7475-7498, 7546-7569, 7614-7637, 7683-7706
//   max(a, b)        Matrix.mm:13459-13474  (std::max: a unless a < b)
//   min(a, b)        Matrix.mm:14757-14781  (std::min: a unless b < a)
//   equal(a, b)      Matrix.mm:14521-14538  (T(1) when a == b, else T(0); decoded there with the
//                    collapsed shape, which gives the same positions for the contiguous result)
// Output element gid is written at out[gid]; per collapsed axis the index is
// rem / sR[i], scaled by sA[i] / sB[i] (stride 0 on broadcast axes).
// cdims == 0 is the scalar case (Matrix.mm:7455-7464).  Integer division by
// zero is undefined in the reference (a trap on x86); callers avoid it.
// ---------------------------------------------------------------------------
int orc_broadcast(int op, int dtype, void* out, const void* a, const void* b, uint32_t cdims, const uint32_t* sR,
                  const uint32_t* sA, const uint32_t* sB, uint64_t total, int threads) {
    if (cdims > kMaxDims || op < 0 || op > 6) return -1;
    const bool ok = with_type(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        const T* pa = static_cast<const T*>(a);
        const T* pb = static_cast<const T*>(b);
        T* pr = static_cast<T*>(out);
        auto apply = [op](T x, T y) -> T {
            switch (op) {
                case 0: return add_wrap<T>(x, y);
                case 1: return sub_wrap<T>(x, y);
                case 2: return mul_wrap<T>(x, y);
                case 3:
                    if constexpr (std::is_same_v<T, bool>) return static_cast<bool>(int(x) / int(y));
                    else return static_cast<T>(x / y);
                case 4: return std::max(x, y);
                case 5: return std::min(x, y);
                default: return x == y ? T(1) : T(0);
            }
        };
        if (cdims == 0) {
            pr[0] = apply(pa[0], pb[0]);
            return;
        }
        parallel_ranges(total, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t gid = lo; gid < hi; ++gid) {
                uint64_t ia = 0, ib = 0, rem = gid;
                for (uint32_t i = 0; i < cdims; ++i) {
                    const uint64_t idx = rem / sR[i];
                    ia += idx * sA[i];
                    ib += idx * sB[i];
                    rem %= sR[i];
                }
                pr[gid] = apply(pa[ia], pb[ib]);
            }
        });
    });
    return ok ? 0 : -1;
}

// ---------------------------------------------------------------------------
// Elementwise exp: Matrix.mm:7014-7063 (CPU branch).  Collapsed two-operand
// metadata: sOut = output strides, sIn = input strides; the element position
// is decoded from the collapsed shape, innermost axis fastest.  Float only.
// ---------------------------------------------------------------------------
int orc_exp(int dtype, void* out, const void* in, uint32_t cdims, const uint32_t* shape, const uint32_t* sOut,
            const uint32_t* sIn, uint64_t total, int threads) {
    if (dtype != kFloat || cdims > kMaxDims) return -1;
    const float* src = static_cast<const float*>(in);
    float* dst = static_cast<float*>(out);
    if (cdims == 0) {
        dst[0] = std::exp(src[0]);
        return 0;
    }
    parallel_ranges(total, threads, [&](uint64_t lo, uint64_t hi) {
        for (uint64_t gid = lo; gid < hi; ++gid) {
            uint64_t si = 0, di = 0, rem = gid;
            for (int i = (int)cdims - 1; i >= 0; --i) {
                const uint64_t idx = rem % shape[i];
                si += idx * sIn[i];
                di += idx * sOut[i];
                rem /= shape[i];
            }
            dst[di] = std::exp(src[si]);
        }
    });
    return 0;
}

// ---------------------------------------------------------------------------
// Elementwise exp / sqrt on Float or Float16 (op 0 exp, 1 sqrt): Matrix.mm:7014-7063 and
// 6870-6925 (CPU branches).  The Float16 element is evaluated in float and rounded back, as
// the reference's float16_t arithmetic does.  Same metadata as orc_exp.
// ---------------------------------------------------------------------------
int orc_unary(int op, int dtype, void* out, const void* in, uint32_t cdims, const uint32_t* shape,
              const uint32_t* sOut, const uint32_t* sIn, uint64_t total, int threads) {
    if ((dtype != kFloat && dtype != kFloat16) || cdims > kMaxDims || op < 0 || op > 1) return -1;
    auto run = [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        const T* src = static_cast<const T*>(in);
        T* dst = static_cast<T*>(out);
        auto f = [op](T x) -> T {
            const float v = static_cast<float>(x);
            return static_cast<T>(op == 0 ? std::exp(v) : std::sqrt(v));
        };
        if (cdims == 0) {
            dst[0] = f(src[0]);
            return;
        }
        parallel_ranges(total, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t gid = lo; gid < hi; ++gid) {
                uint64_t si = 0, di = 0, rem = gid;
                for (int i = (int)cdims - 1; i >= 0; --i) {
                    const uint64_t idx = rem % shape[i];
                    si += idx * sIn[i];
                    di += idx * sOut[i];
                    rem /= shape[i];
                }
                dst[di] = f(src[si]);
            }
        });
    };
    if (dtype == kFloat) run((float*)nullptr);
    else run((_Float16*)nullptr);
    return 0;
}

// ---------------------------------------------------------------------------
// astype / copy: copyCPUinplaceTypeCasted, matrix.h:1474-1544, over
// collapse_dims(in.shape, out.strides, in.strides) (matrix.h:1481); element
// conversion dtype_cast (cast_elem above).  The loops there walk the collapsed
// shape innermost axis fastest; gid is decoded the same way here.
// ---------------------------------------------------------------------------
// (GCC 13 at -O3 miscompiles vectorised Float16 <-> BFloat16 conversion loops, storing the source
// bits unconverted; the loop vectoriser is kept off here.)
#pragma GCC push_options
#pragma GCC optimize("no-tree-loop-vectorize")
int orc_astype(int dst_dtype, int src_dtype, void* out, const void* in, uint32_t cdims, const uint32_t* shape,
               const uint32_t* sOut, const uint32_t* sIn, uint64_t total, int threads) {
    if (cdims > kMaxDims) return -1;
    bool inner_ok = false;
    const bool ok = with_type(dst_dtype, [&](auto* dtag) {
        using D = std::remove_pointer_t<decltype(dtag)>;
        inner_ok = with_type(src_dtype, [&](auto* stag) {
            using S = std::remove_pointer_t<decltype(stag)>;
            const S* src = static_cast<const S*>(in);
            D* dst = static_cast<D*>(out);
            if (cdims == 0) {
                dst[0] = cast_elem<D, S>(src[0]);
                return;
            }
            parallel_ranges(total, threads, [&](uint64_t lo, uint64_t hi) {
                for (uint64_t gid = lo; gid < hi; ++gid) {
                    uint64_t si = 0, di = 0, rem = gid;
                    for (int i = (int)cdims - 1; i >= 0; --i) {
                        const uint64_t idx = rem % shape[i];
                        si += idx * sIn[i];
                        di += idx * sOut[i];
                        rem /= shape[i];
                    }
                    dst[di] = cast_elem<D, S>(src[si]);
                }
            });
        });
    });
    return ok && inner_ok ? 0 : -1;
}
#pragma GCC pop_options

// ---------------------------------------------------------------------------
// make_pointwise's collapse: Matrix.mm:13537-13555.  Output axes outermost
// first; extent-1 axes are skipped; an axis folds into the last kept one when
// the merged extent stays <= INT32_MAX and every input's kept stride equals
// its stride here times this extent (compared in 64 bits); the kept axis then
// takes this axis' strides.  in_strides: n rows of out_dims entries; outputs:
// the collapsed shape (kMaxDims entries) and n rows of kMaxDims strides.
// Returns the collapsed rank, or UINT32_MAX where the reference throws.
// ---------------------------------------------------------------------------
uint32_t orc_pointwise_collapse(const uint32_t* out_shape, uint32_t out_dims, const uint32_t* in_strides,
                                uint32_t n, uint32_t* cshape, uint32_t* cstrides) {
    if (out_dims > kMaxDims || n > 3) return UINT32_MAX;
    uint64_t count = 1;
    for (uint32_t d = 0; d < out_dims; ++d) {
        if (out_shape[d] && count > UINT32_MAX / out_shape[d]) return UINT32_MAX;
        count *= out_shape[d];
    }
    std::fill(cshape, cshape + kMaxDims, 0u);
    std::fill(cstrides, cstrides + n * kMaxDims, 0u);
    uint32_t dims = 0;
    if (!count) return 0;
    for (uint32_t d = 0; d < out_dims; ++d) {
        if (out_shape[d] == 1) continue;
        bool merge = dims > 0 && uint64_t(cshape[dims - 1]) * out_shape[d] <= INT32_MAX;
        if (merge) {
            for (uint32_t i = 0; i < n; ++i) {
                if (uint64_t(cstrides[i * kMaxDims + dims - 1]) != uint64_t(in_strides[i * out_dims + d]) * out_shape[d]) {
                    merge = false;
                    break;
                }
            }
        }
        const uint32_t target = merge ? dims - 1 : dims++;
        if (merge) cshape[target] *= out_shape[d];
        else cshape[target] = out_shape[d];
        for (uint32_t i = 0; i < n; ++i) cstrides[i * kMaxDims + target] = in_strides[i * out_dims + d];
    }
    return dims;
}

// ---------------------------------------------------------------------------
// The make_pointwise family's CPU backends: op 0 greater (Matrix.mm:13803-13874),
// 1 less (13876-13947), 2 logical_and (13949-14020), 3 where (14022-14103),
// 4 floor (13741-13801), 5 full (14105-14165), 6 arctan2 (13608-13678),
// 7 arcsin (13680-13738).  The output is contiguous and written in order
// (dst[i++]); input k is read at sum idx * strides[k][axis] (kMaxDims entries
// per row).  dtype is the inputs' common dtype (Bool for logical_and; the dtype
// of a and b for where, whose cond is Bool; Float for arctan2 / arcsin, which
// write std::atan2(float(a), float(b)) / std::asin(float(x)) as float).
// Greater, less and logical_and write bool.  cdims == 0 is one element at offset 0.
// ---------------------------------------------------------------------------
int orc_pointwise(int op, int dtype, void* out, const void* const* inputs, uint32_t n, uint32_t cdims,
                  const uint32_t* shape, const uint32_t* strides, uint64_t total, int threads) {
    static const uint32_t kArity[] = {2, 2, 2, 3, 1, 1, 2, 1};
    if (op < 0 || op > 7 || n != kArity[op] || cdims > kMaxDims) return -1;
    if (op == 2 && dtype != kBool) return -1;
    const bool ok = with_type(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        auto offset = [&](uint64_t gid, uint32_t k) {
            uint64_t off = 0, rem = gid;
            for (int i = (int)cdims - 1; i >= 0; --i) {
                off += (rem % shape[i]) * strides[k * kMaxDims + i];
                rem /= shape[i];
            }
            return off;
        };
        parallel_ranges(cdims == 0 ? 1 : total, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t gid = lo; gid < hi; ++gid) {
                if (op == 0 || op == 1 || op == 2) {
                    const T* a = static_cast<const T*>(inputs[0]);
                    const T* b = static_cast<const T*>(inputs[1]);
                    const T x = a[offset(gid, 0)], y = b[offset(gid, 1)];
                    bool r;
                    if (op == 0) r = x > y;
                    else if (op == 1) r = x < y;
                    else r = bool(x) && bool(y);
                    static_cast<bool*>(out)[gid] = r;
                } else if (op == 6) {
                    const T x = static_cast<const T*>(inputs[0])[offset(gid, 0)];
                    const T y = static_cast<const T*>(inputs[1])[offset(gid, 1)];
                    static_cast<float*>(out)[gid] = std::atan2(static_cast<float>(x), static_cast<float>(y));
                } else if (op == 7) {
                    const T x = static_cast<const T*>(inputs[0])[offset(gid, 0)];
                    static_cast<float*>(out)[gid] = std::asin(static_cast<float>(x));
                } else if (op == 3) {
                    const bool* c = static_cast<const bool*>(inputs[0]);
                    const T* a = static_cast<const T*>(inputs[1]);
                    const T* b = static_cast<const T*>(inputs[2]);
                    static_cast<T*>(out)[gid] = c[offset(gid, 0)] ? a[offset(gid, 1)] : b[offset(gid, 2)];
                } else {
                    const T x = static_cast<const T*>(inputs[0])[offset(gid, 0)];
                    if (op == 5 || std::is_integral_v<T>) static_cast<T*>(out)[gid] = x;
                    else static_cast<T*>(out)[gid] = cast_elem<T, float>(std::floor(static_cast<float>(x)));
                }
            }
        });
    });
    return ok ? 0 : -1;
}

// ---------------------------------------------------------------------------
// arange's CPU backend (Matrix.mm:14167-14180): out[i] = start + i * step in the
// output type T, for i < count; integers through uint64 arithmetic cast back,
// float-likes as float(start) + float(i) * float(step) converted by dtype_cast.
// start and step are one element of T each.  Bool is refused (-1), as arange does.
// ---------------------------------------------------------------------------
int orc_arange(int dtype, void* out, const void* start, const void* step, uint64_t count) {
    if (dtype == kBool) return -1;
    const bool ok = with_type(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        const T a = *static_cast<const T*>(start), b = *static_cast<const T*>(step);
        T* dst = static_cast<T*>(out);
        for (uint64_t i = 0; i < count; ++i) {
            if constexpr (std::is_integral_v<T>) dst[i] = static_cast<T>(uint64_t(a) + uint64_t(i) * uint64_t(b));
            else dst[i] = cast_elem<T, float>(float(a) + float(i) * float(b));
        }
    });
    return ok ? 0 : -1;
}

}  // extern "C"
