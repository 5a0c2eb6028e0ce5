// Axis reductions (Sum, Max, Min, ArgMax, ArgMin) for sm_100a.
//
// Replaces the reference's Metal reduction kernels (ComputeShaders/Sum.metal, Max.metal,
// Min.metal, ArgMax.metal, ArgMin.metal) behind the METAL branch of matrix::sum / max / min /
// argmax / argmin (Matrix.mm:14812-16458).  The results follow the reference CPU eval:
//   Sum     T accumulator from 0; integer sums wrap (accumulated in the unsigned type of the
//           accumulator width, which is the same value modulo 2^bits); float sums agree
//           within rounding (tree order instead of sequential order).
//   Max/Min start from dtype_lowest / dtype_max; an element replaces the running value only
//           when strictly greater / smaller, so NaN never wins and among equal extremes the
//           first one is kept (this matters for floats: -0.0 vs +0.0).
//   ArgMax/ArgMin (value, index) with the same strict rule; the lowest index wins ties; 0 when
//           no element beats the initial value.  Output int32.
// Float Max / Min therefore carry the element index too: a (value, index) pair reduction is
// the one order-free formulation of "first among equals", which is what lets the kernels
// read elements in any order (vector lanes, interleaved rows, split axes).
//
// Three kernels, chosen on the host from the collapsed metadata:
//   rows    reduce_stride == 1: each output reduces a contiguous run.  A warp (G = 32) or a
//           256-thread CTA (G = 256) owns a (row, split) unit and streams it with 128-bit
//           loads (scalar head / tail around the 16-byte aligned body).
//   cols    reduce_stride != 1 and the innermost output axis is contiguous in the input: a
//           warp spans 32 x V consecutive outputs with one vector load per lane per reduced row
//           (V x sizeof(T) = 16 bytes, fewer for the narrow types), the CTA's 8 warps interleave the reduced rows, and CTAs
//           split the reduced axis when there are too few outputs to fill 148 SMs.
//   generic anything else (non-row-major output strides, short rows, odd layouts): one
//           thread per output walking its run, exactly like the reference CPU loop.
// When the axis is split across CTAs, per-split partials go to the thread's workspace and a
// second kernel merges them in a fixed order (split order for a few splits; lane-strided runs and a
// warp shuffle tree for many), so results are deterministic for a given split.
#include <algorithm>
#include <map>
#include <mutex>

#include <atomic>

#include "elementwise.cuh"

namespace mtxc {
namespace {

constexpr int kBlock = 256;
constexpr int kUnroll = 4;
constexpr uint32_t kSplitWaves = 4;

// ------------------------------------------------------------------------------------------
// Reducer definitions
// ------------------------------------------------------------------------------------------
template <typename T>
struct Pair {
    T v;
    int32_t i;
};
template <typename S>
struct IsPair : std::false_type {};
template <typename T>
struct IsPair<Pair<T>> : std::true_type {};

template <typename T>
__device__ __forceinline__ T shfl_xor(T v, int mask) {
    if constexpr (sizeof(T) == 8) {
        unsigned long long x;
        memcpy(&x, &v, 8);
        x = __shfl_xor_sync(0xffffffffu, x, mask);
        T r;
        memcpy(&r, &x, 8);
        return r;
    } else {
        // 1-, 2- and 4-byte values travel in the low bytes of a 32-bit register
        unsigned x = 0;
        memcpy(&x, &v, sizeof(T));
        x = __shfl_xor_sync(0xffffffffu, x, mask);
        T r;
        memcpy(&r, &x, sizeof(T));
        return r;
    }
}

// Where a reduction writes: values (T, or int32 indices for ArgMax / ArgMin) and, for the
// (value, index) pair ops, the indices as well.
struct Out {
    void* v;
    int32_t* i;
    uint32_t n = 0;  // reduced length (the divisor of a mean)
};

// Internal op codes beyond the public ones: ArgMax / ArgMin writing both the extreme value and its
// first index (mtxc_reduce_pair), and the fused statistics of mtxc_reduce_stat.
constexpr int kPairMax = 5;
constexpr int kPairMin = 6;
constexpr int kStatMean = 7;
constexpr int kStatRms = 8;
constexpr int kStatNorm = 9;

// Columns per lane of the column kernel: 16 bytes' worth, read with one 16-byte load per reduced row;
// when the operand is not 16-byte aligned, the 1- and 2-byte types fall back to 4-byte lanes.
template <int OP, typename T>
constexpr int col_vec() {
    return 16 / (int)sizeof(T);
}
template <typename T>
constexpr int col_vec_narrow() {
    return sizeof(T) <= 2 ? 4 / (int)sizeof(T) : 1;
}

template <int OP, typename T>
struct Reducer;

// packed lanes of a vector-folding reducer: one 16-byte vector's worth of partial results
struct Lanes {
    uint32_t w[4];
};

// Sum: float-likes accumulate in fp32 (rounded to T once, at the end); integers in the unsigned
// type of the accumulator width (wrap-around, as the reference's T accumulator); Bool as C++ bool
// does, where `acc += x` is a logical or.
template <typename T>
struct Reducer<MTXC_REDUCE_SUM, T> {
    using State = typename Traits<T>::Acc;
    __device__ static State init() { return State(0); }
    __device__ static void fold(State& s, T v, uint32_t) {
        if constexpr (Traits<T>::kFloat) s = __fadd_rn(s, to_float(v));
        else if constexpr (Traits<T>::kBool) s |= (State)(uint8_t)v;
        else s = (State)(s + (State)v);
    }
    __device__ static void merge(State& s, const State& o) {
        if constexpr (Traits<T>::kFloat) s = __fadd_rn(s, o);
        else if constexpr (Traits<T>::kBool) s |= o;
        else s = (State)(s + o);
    }
    __device__ static State shfl(const State& s, int m) { return shfl_xor(s, m); }
    // The 1-byte types fold whole 16-byte vectors into a packed state of four words, reduced into a
    // State once per segment: dp4a adds four bytes per instruction into each word (the wrap-around
    // sum is the same modulo 2^bits), a Bool sum is an or of the words.
    static constexpr bool kVecFold = sizeof(T) == 1;
    __device__ static Lanes vec_init() { return Lanes{}; }
    __device__ static void vec_fold(Lanes& p, const Vec16<T>& x) {
        uint32_t w[4];
        memcpy(w, &x, 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (Traits<T>::kBool) p.w[i] |= w[i];
            else if constexpr (std::is_signed_v<T>) p.w[i] = (uint32_t)__dp4a((int)w[i], 0x01010101, (int)p.w[i]);
            else p.w[i] = __dp4a(w[i], 0x01010101u, p.w[i]);
        }
    }
    __device__ static void vec_finish(State& s, const Lanes& p) {
        if constexpr (Traits<T>::kBool) s |= (p.w[0] | p.w[1] | p.w[2] | p.w[3]) != 0u;
        else s = (State)(s + (State)(p.w[0] + p.w[1] + p.w[2] + p.w[3]));
    }
    // Column kernel, 1-byte types: a lane's 16 columns accumulate in the 16-bit halves of eight words
    // (even bytes, odd bytes), masked back to their low byte every 256 rows before a half can carry into
    // its neighbour.  The low byte is the sum modulo 2^8, all that the 1-byte result keeps of the
    // wrap-around sum.  Bool ors the words.
    static constexpr bool kColSimd = sizeof(T) == 1;
    struct ColState {
        uint32_t e[4], o[4];
        uint32_t n;
    };
    __device__ static ColState col_init(uint32_t, uint32_t, uint32_t = 0) { return ColState{}; }
    __device__ static void col_fold(ColState& c, const uint32_t (&w)[4], uint32_t) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (Traits<T>::kBool) {
                c.e[i] |= w[i];
            } else {
                c.e[i] += w[i] & 0x00ff00ffu;
                c.o[i] += __byte_perm(w[i], 0u, 0x4341u);  // bytes 1 and 3 into the halves' low bytes
            }
        }
        if constexpr (!Traits<T>::kBool) {
            if (++c.n == 256u) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    c.e[i] &= 0x00ff00ffu;
                    c.o[i] &= 0x00ff00ffu;
                }
                c.n = 0;
            }
        }
    }
    __device__ static void col_finish(ColState& c, State (&st)[16]) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int i = j / 4, b = j % 4;
            if constexpr (Traits<T>::kBool) st[j] = (State)((c.e[i] >> (8 * b)) & 0xffu);
            else st[j] = (State)(((b % 2 ? c.o[i] : c.e[i]) >> (16 * (b / 2))) & 0xffu);
        }
    }
    __device__ static void store(const Out& o, uint64_t gid, const State& s) {
        if constexpr (Traits<T>::kFloat) static_cast<T*>(o.v)[gid] = from_float<T>(s);
        else if constexpr (Traits<T>::kBool) static_cast<T*>(o.v)[gid] = mbool(s != 0);
        else static_cast<T*>(o.v)[gid] = (T)s;
    }
};

// Extremum with index (float-likes for Max / Min; every type for ArgMax / ArgMin).  The half types keep
// the running value in float: the widening is exact, so comparisons, NaN and ties are unchanged, and each
// element is converted once instead of at every comparison.
template <typename T, bool kMax>
struct PairExtremum {
    using V = std::conditional_t<Traits<T>::kFloat, float, T>;
    using State = Pair<V>;
    __device__ static V widen(T v) {
        if constexpr (Traits<T>::kFloat) return to_float(v);
        else return v;
    }
    __device__ static T narrow(V v) {
        if constexpr (Traits<T>::kFloat) return from_float<T>(v);  // exact: v came from a T
        else return v;
    }
    __device__ static State init() { return State{widen(kMax ? lowest_value<T>() : highest_value<T>()), 0}; }
    __device__ static bool beats(V a, V b) { return kMax ? less(b, a) : less(a, b); }
    __device__ static void fold(State& s, T x, uint32_t i) {
        const V v = widen(x);
        if (beats(v, s.v)) {
            s.v = v;
            s.i = (int32_t)i;
        }
    }
    __device__ static void merge(State& s, const State& o) {
        if (beats(o.v, s.v) || (equal(o.v, s.v) && o.i < s.i)) s = o;
    }
    __device__ static State shfl(const State& s, int m) { return State{shfl_xor(s.v, m), shfl_xor(s.i, m)}; }

    // Column kernel (and the row kernel's lanes), 1- and 2-byte types.  A lane's 16 bytes of columns
    // are folded without per-element branches in one of two ways.
    //
    // Integers and Bool (keyed): each element and its row form one 32-bit key, the element's bits on
    // top (24 or 16 bits up) and a row part below that decreases with the row for Max (increases for
    // Min), so one integer max (min) of keys -- signed for the signed types, unsigned for the others
    // and Bool -- picks the larger value and, among equal values, the earlier row: exactly the strict
    // "first index wins" rule.  Building a key is one byte permute; two rows fold with one 3-input
    // max (min).  The row part counts the lane's rows within a chunk (at most 2^24 - 2 or 2^16 - 2
    // rows); at a chunk's end the lanes whose best came from it turn the count back into a row index,
    // and their key's row part becomes the carried mark, which beats (loses to) every later row of
    // the same value.  The initial key (dtype_lowest / dtype_max with the row part that loses every
    // tie) marks a lane that saw no row.
    //
    // The half types (packed): the lane's best values stay packed in four words; per reduced row, one
    // SIMD compare per word (as the floats they widen to) gives the lanes the row beats (strictly, so
    // the first row of a tie is kept; NaN never beats), the row's bits replace the best in exactly
    // those lanes, and the row's number within the current chunk of rows (1-based, 16 bits) is merged
    // into the packed 16-bit "row of the best" lanes there (a row that beats no lane skips both).  A
    // chunk ends after 65,535 rows or at the end of the lane's rows: lanes that won in it turn their
    // chunk number back into a row index.
    //
    // Either way every index stays exact whatever the length.
    static constexpr bool kColSimd = sizeof(T) <= 2;
    static constexpr int kLanes = 16 / (int)sizeof(T);
    static constexpr bool kKeyed = kColSimd && !Traits<T>::kFloat;
    // the key layout (a nested class: instantiated only with the keyed folds that use it)
    struct Key {
        static constexpr int kShift = 32 - 8 * (int)sizeof(T);
        static constexpr uint32_t kLow = (1u << kShift) - 1u;         // the row part of a key
        static constexpr uint32_t kCarried = kMax ? kLow : 0u;          // best from an earlier chunk
        static constexpr uint32_t kUnset = kMax ? 0u : kLow;            // no row yet
        // int32 words from one carried index to the next: the index fields of consecutive (value, index) states
        static constexpr int kIdxStride = (int)(sizeof(Pair<V>) / sizeof(int32_t));
    };
    struct KeyState {
        uint32_t key[kLanes];
        // row indices of carried bests (lane j at idx[j * Key::kIdxStride]): memory of the caller's choosing,
        // written only at a chunk's end and read at the finish -- the column kernel points it at the index
        // fields of the thread's own shared-memory staging slots, which are free until its epilogue, so the
        // indices hold no registers through the loop
        int32_t* idx;
        uint32_t n;                // rows of the current chunk so far
        uint32_t row;              // last row folded
        uint32_t step;             // distance between the lane's consecutive rows
        uint32_t limit;            // rows per chunk (at most Key::kLow - 1, so row parts stay clear of both marks)
        uint32_t lane_stride;      // index distance between neighbouring lanes (rows: 1, columns: 0)
    };
    __device__ static uint32_t key_bits(T v) {
        uint32_t b = 0;
        memcpy(&b, &v, sizeof(T));
        return b << Key::kShift;
    }
    __device__ static uint32_t key_ext(uint32_t a, uint32_t b) {
        if constexpr (std::is_signed_v<T>) return (uint32_t)(kMax ? max((int)a, (int)b) : min((int)a, (int)b));
        else return kMax ? umax(a, b) : umin(a, b);
    }
    __device__ static uint32_t key_ext3(uint32_t a, uint32_t b, uint32_t c) {
        if constexpr (std::is_signed_v<T>)
            return (uint32_t)(kMax ? __vimax3_s32((int)a, (int)b, (int)c) : __vimin3_s32((int)a, (int)b, (int)c));
        else return kMax ? __vimax3_u32(a, b, c) : __vimin3_u32(a, b, c);
    }
    // the key of lane j of the packed row w: its element on top, the row part rk below
    __device__ static uint32_t key_of(const uint32_t (&w)[4], int j, uint32_t rk) {
        if constexpr (sizeof(T) == 1) return __byte_perm(w[j / 4], rk, 0x0654u | ((uint32_t)(j % 4) << 12));
        else return __byte_perm(w[j / 2], rk, 0x0054u | ((uint32_t)(j % 2) << 9) | ((uint32_t)(j % 2 * 2 + 1) << 12));
    }
    __device__ static uint32_t row_part(uint32_t n) { return kMax ? (Key::kLow - 1u) - n : n + 1u; }
    __device__ static KeyState col_init_keyed(uint32_t step, uint32_t limit, uint32_t lane_stride, int32_t* idx) {
        KeyState c;
        const uint32_t k0 = key_bits(kMax ? lowest_value<T>() : highest_value<T>()) | Key::kUnset;
#pragma unroll
        for (int j = 0; j < kLanes; ++j) {
            c.key[j] = k0;  // idx needs no initial value: it is read only for lanes that a flush carried
        }
        c.idx = idx;
        c.n = 0;
        c.row = 0;
        c.step = step;
        c.limit = min(limit, Key::kLow - 1u);
        c.lane_stride = lane_stride;
        return c;
    }
    __device__ static void col_flush(KeyState& c) {
#pragma unroll
        for (int j = 0; j < kLanes; ++j) {
            const uint32_t low = c.key[j] & Key::kLow;
            if (low != Key::kCarried && low != Key::kUnset) {
                const uint32_t cnt = kMax ? (Key::kLow - 1u) - low : low - 1u;  // the row's count in this chunk
                c.idx[j * Key::kIdxStride] = (int32_t)(c.row - (c.n - 1u - cnt) * c.step + (uint32_t)j * c.lane_stride);
                c.key[j] = (c.key[j] & ~Key::kLow) | Key::kCarried;
            }
        }
        c.n = 0;
    }
    __device__ static void col_fold(KeyState& c, const uint32_t (&w)[4], uint32_t row) {
        const uint32_t rk = row_part(c.n);
#pragma unroll
        for (int j = 0; j < kLanes; ++j) c.key[j] = key_ext(c.key[j], key_of(w, j, rk));
        c.n += 1;
        c.row = row;
        if (c.n == c.limit) col_flush(c);
    }
    // two consecutive rows of the lane (row_b = row_a + step)
    __device__ static void col_fold2(KeyState& c, const uint32_t (&wa)[4], const uint32_t (&wb)[4], uint32_t row_a,
                                     uint32_t row_b) {
        if (c.n + 2u > c.limit) {
            col_fold(c, wa, row_a);
            col_fold(c, wb, row_b);
            return;
        }
        const uint32_t ra = row_part(c.n), rb = row_part(c.n + 1u);
#pragma unroll
        for (int j = 0; j < kLanes; ++j) c.key[j] = key_ext3(c.key[j], key_of(wa, j, ra), key_of(wb, j, rb));
        c.n += 2;
        c.row = row_b;
        if (c.n == c.limit) col_flush(c);
    }
    __device__ static void col_finish(KeyState& c, State (&st)[kLanes]) {
        if (c.n) col_flush(c);
#pragma unroll
        for (int j = 0; j < kLanes; ++j) {
            if ((c.key[j] & Key::kLow) == Key::kUnset) {
                st[j] = init();
            } else {
                T v;
                const uint32_t b = c.key[j] >> Key::kShift;
                memcpy(&v, &b, sizeof(T));  // little-endian: the element's bits are the low bytes of b
                st[j] = State{widen(v), c.idx[j * Key::kIdxStride]};
            }
        }
    }

    struct PackedState {
        Lanes best;
        uint32_t won[kLanes / 2];  // 16-bit lanes: chunk row number of the lane's best, 0 = none yet
        int32_t idx[kLanes];       // row index of the best as of the last finished chunk
        uint32_t n;                // rows of the current chunk so far
        uint32_t row;              // last row folded
        uint32_t step;             // distance between the lane's consecutive rows
        uint32_t limit;            // rows per chunk (at most 65,535)
        uint32_t lane_stride;      // index distance between neighbouring lanes (rows: 1, columns: 0)
    };
    __device__ static uint32_t simd_beats(uint32_t x, uint32_t b) {  // all ones in the lanes where x beats b
        if constexpr (std::is_same_v<T, __half>) {
            __half2 hx, hb;
            memcpy(&hx, &x, 4);
            memcpy(&hb, &b, 4);
            return kMax ? __hgt2_mask(hx, hb) : __hlt2_mask(hx, hb);
        } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
            __nv_bfloat162 hx, hb;
            memcpy(&hx, &x, 4);
            memcpy(&hb, &b, 4);
            return kMax ? __hgt2_mask(hx, hb) : __hlt2_mask(hx, hb);
        } else if constexpr (sizeof(T) == 1 && std::is_signed_v<T>) {
            return kMax ? __vcmpgts4(x, b) : __vcmplts4(x, b);
        } else if constexpr (sizeof(T) == 1) {
            return kMax ? __vcmpgtu4(x, b) : __vcmpltu4(x, b);
        } else if constexpr (std::is_signed_v<T>) {
            return kMax ? __vcmpgts2(x, b) : __vcmplts2(x, b);
        } else {
            return kMax ? __vcmpgtu2(x, b) : __vcmpltu2(x, b);
        }
    }
    using ColState = std::conditional_t<kKeyed, KeyState, PackedState>;
    // the half types' state (the keyed types start with col_init_keyed, which also takes the carried
    // indices' storage)
    __device__ static PackedState col_init(uint32_t step, uint32_t limit, uint32_t lane_stride = 0) {
        return col_init_packed(step, limit, lane_stride);
    }
    __device__ static PackedState col_init_packed(uint32_t step, uint32_t limit, uint32_t lane_stride) {
        PackedState c;
        Vec16<T> v;
#pragma unroll
        for (int j = 0; j < kLanes; ++j) {
            v.v[j] = kMax ? lowest_value<T>() : highest_value<T>();
            c.idx[j] = 0;
        }
        memcpy(&c.best, &v, 16);
#pragma unroll
        for (int i = 0; i < kLanes / 2; ++i) c.won[i] = 0;
        c.n = 0;
        c.row = 0;
        c.step = step;
        c.limit = limit;
        c.lane_stride = lane_stride;
        return c;
    }
    // lanes that won in the current chunk take the row index of their last win; the chunk restarts
    __device__ static void col_flush(PackedState& c) {
#pragma unroll
        for (int j = 0; j < kLanes; ++j) {
            const uint32_t t = (c.won[j / 2] >> (16 * (j % 2))) & 0xffffu;
            if (t != 0) c.idx[j] = (int32_t)(c.row - (c.n - t) * c.step + (uint32_t)j * c.lane_stride);
        }
#pragma unroll
        for (int i = 0; i < kLanes / 2; ++i) c.won[i] = 0;
        c.n = 0;
    }
    __device__ static void col_fold(PackedState& c, const uint32_t (&w)[4], uint32_t row) {
        c.n += 1;
        c.row = row;
        const uint32_t t2 = c.n * 0x00010001u;  // the chunk row number in both 16-bit halves
        uint32_t m[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) m[i] = simd_beats(w[i], c.best.w[i]);
        // a row that beats no lane changes nothing (the common case once the columns' extremes are
        // found, e.g. Bool after its first true)
        if ((m[0] | m[1] | m[2] | m[3]) != 0u) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                c.best.w[i] = (c.best.w[i] & ~m[i]) | (w[i] & m[i]);
                if constexpr (sizeof(T) == 1) {
                    // byte lanes (4i .. 4i+3) -> the 16-bit lanes of won[2i] and won[2i + 1]
                    const uint32_t lo = __byte_perm(m[i], 0, 0x1100), hi = __byte_perm(m[i], 0, 0x3322);
                    c.won[2 * i] = (c.won[2 * i] & ~lo) | (t2 & lo);
                    c.won[2 * i + 1] = (c.won[2 * i + 1] & ~hi) | (t2 & hi);
                } else {
                    c.won[i] = (c.won[i] & ~m[i]) | (t2 & m[i]);
                }
            }
        }
        if (c.n == c.limit) col_flush(c);
    }
    __device__ static void col_finish(PackedState& c, State (&st)[kLanes]) {
        col_flush(c);
        Vec16<T> v;
        memcpy(&v, &c.best, 16);
#pragma unroll
        for (int j = 0; j < kLanes; ++j) st[j] = State{widen(v.v[j]), c.idx[j]};
    }
};

// Integer and Bool Max / Min: equal values are indistinguishable, so no index is needed.
template <typename T, bool kMax>
struct ValueExtremum {
    using State = T;
    __device__ static State init() { return kMax ? lowest_value<T>() : highest_value<T>(); }
    __device__ static void fold(State& s, T v, uint32_t) {
        if (kMax ? less(s, v) : less(v, s)) s = v;
    }
    // 1- and 2-byte integers and Bool (its bytes compare unsigned) fold 16-byte vectors into a packed
    // state of four words with the per-byte / per-half SIMD max / min, whose lanes are reduced into a
    // State once per segment
    static constexpr bool kVecFold = sizeof(T) <= 2;
    __device__ static uint32_t ext2(uint32_t a, uint32_t b) {
        if constexpr (sizeof(T) == 1 && std::is_signed_v<T>) return kMax ? __vmaxs4(a, b) : __vmins4(a, b);
        else if constexpr (sizeof(T) == 1) return kMax ? __vmaxu4(a, b) : __vminu4(a, b);
        else if constexpr (std::is_signed_v<T>) return kMax ? __vmaxs2(a, b) : __vmins2(a, b);
        else return kMax ? __vmaxu2(a, b) : __vminu2(a, b);
    }
    __device__ static Lanes vec_init() {
        Vec16<T> x;
#pragma unroll
        for (int j = 0; j < Vec16<T>::N; ++j) x.v[j] = init();
        Lanes p;
        memcpy(&p, &x, 16);
        return p;
    }
    __device__ static void vec_fold(Lanes& p, const Vec16<T>& x) {
        uint32_t w[4];
        memcpy(w, &x, 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) p.w[i] = ext2(p.w[i], w[i]);
    }
    __device__ static void vec_finish(State& s, const Lanes& p) {
        uint32_t m = ext2(ext2(p.w[0], p.w[1]), ext2(p.w[2], p.w[3]));
        m = ext2(m, m >> 16);                               // low lane: the extreme of lanes (0, 2) and (1, 3)
        if constexpr (sizeof(T) == 1) m = ext2(m, m >> 8);  // low byte: the extreme of all four
        if constexpr (sizeof(T) == 1) fold(s, (T)(uint8_t)m, 0);
        else fold(s, (T)(uint16_t)m, 0);
    }
    // column kernel: the 16 columns of a lane fold as one packed vector
    static constexpr bool kColSimd = kVecFold;
    using ColState = Lanes;
    __device__ static Lanes col_init(uint32_t, uint32_t, uint32_t = 0) { return vec_init(); }
    __device__ static void col_fold(Lanes& p, const uint32_t (&w)[4], uint32_t) {
#pragma unroll
        for (int i = 0; i < 4; ++i) p.w[i] = ext2(p.w[i], w[i]);
    }
    __device__ static void col_finish(Lanes& p, State (&st)[Vec16<T>::N]) {
        Vec16<T> v;
        memcpy(&v, &p, 16);
#pragma unroll
        for (int j = 0; j < Vec16<T>::N; ++j) st[j] = v.v[j];
    }
    __device__ static void merge(State& s, const State& o) { fold(s, o, 0); }
    __device__ static State shfl(const State& s, int m) { return shfl_xor(s, m); }
    __device__ static void store(const Out& o, uint64_t gid, const State& s) { static_cast<T*>(o.v)[gid] = s; }
};

template <typename T, bool kMax>
using ExtremumOf = std::conditional_t<Traits<T>::kFloat, PairExtremum<T, kMax>, ValueExtremum<T, kMax>>;

template <typename T>
struct Reducer<MTXC_REDUCE_MAX, T> : ExtremumOf<T, true> {
    using Base = ExtremumOf<T, true>;
    __device__ static void store(const Out& o, uint64_t gid, const typename Base::State& s) {
        if constexpr (Traits<T>::kFloat) static_cast<T*>(o.v)[gid] = Base::narrow(s.v);
        else static_cast<T*>(o.v)[gid] = s;
    }
};
template <typename T>
struct Reducer<MTXC_REDUCE_MIN, T> : ExtremumOf<T, false> {
    using Base = ExtremumOf<T, false>;
    __device__ static void store(const Out& o, uint64_t gid, const typename Base::State& s) {
        if constexpr (Traits<T>::kFloat) static_cast<T*>(o.v)[gid] = Base::narrow(s.v);
        else static_cast<T*>(o.v)[gid] = s;
    }
};
template <typename T>
struct Reducer<MTXC_REDUCE_ARGMAX, T> : PairExtremum<T, true> {
    using Base = PairExtremum<T, true>;
    __device__ static void store(const Out& o, uint64_t gid, const typename Base::State& s) {
        static_cast<int32_t*>(o.v)[gid] = s.i;
    }
};
template <typename T>
struct Reducer<MTXC_REDUCE_ARGMIN, T> : PairExtremum<T, false> {
    using Base = PairExtremum<T, false>;
    __device__ static void store(const Out& o, uint64_t gid, const typename Base::State& s) {
        static_cast<int32_t*>(o.v)[gid] = s.i;
    }
};
// Max / Min value and its first index in one pass: exactly the Max and ArgMax (Min and ArgMin)
// results, since a (value, index) state that was never updated holds (initial value, 0).
template <typename T>
struct Reducer<kPairMax, T> : PairExtremum<T, true> {
    using Base = PairExtremum<T, true>;
    __device__ static void store(const Out& o, uint64_t gid, const typename Base::State& s) {
        static_cast<T*>(o.v)[gid] = Base::narrow(s.v);
        o.i[gid] = s.i;
    }
};
template <typename T>
struct Reducer<kPairMin, T> : PairExtremum<T, false> {
    using Base = PairExtremum<T, false>;
    __device__ static void store(const Out& o, uint64_t gid, const typename Base::State& s) {
        static_cast<T*>(o.v)[gid] = Base::narrow(s.v);
        o.i[gid] = s.i;
    }
};

// ------------------------------------------------------------------------------------------
// Fused statistics: mean = sum / (float)n, rms = sqrt(mean(x * x)), norm = sqrt(sum(x * x)), as
// the reference composes them from its primitives (Matrix.mm:15220-15276), in one pass.
//   * x * x is the reference's element product in T: fp32 product rounded once to T for the
//     float-likes, the wrapped product for integers, x itself for Bool.
//   * the sum is the Sum reducer's (fp32 for float-likes, wrapping integer, logical-or Bool),
//     rounded to T once: the SumPrimitive's output.
//   * the division is `sum / (float)n` with the scalar in scalar_operand_type's dtype (matrix.h:
//     1815-1846): Float and BFloat16 keep their type (the divisor rounded to it), Float16 keeps its
//     type when n <= 65504, everything else divides in Float after astype.  One rounded division.
//   * sqrt runs in promote_types(type, Float16) (Matrix.mm:6798-6811): Float16 stays half, Bool
//     becomes half, BFloat16 and the integers become Float.  One correctly rounded square root.
// ------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T square_in_type(T v) {
    if constexpr (std::is_same_v<T, float>) return __fmul_rn(v, v);
    else if constexpr (Traits<T>::kFloat) return from_float<T>(__fmul_rn(to_float(v), to_float(v)));
    else if constexpr (Traits<T>::kBool) return v;
    else {
        using W = std::conditional_t<(sizeof(T) <= 4), uint32_t, uint64_t>;
        return (T)(W)((W)v * (W)v);
    }
}

// float value of an element (integers round to nearest, Bool is 0 / 1)
template <typename T>
__device__ __forceinline__ float as_float(T v) {
    if constexpr (Traits<T>::kFloat) return to_float(v);
    else if constexpr (Traits<T>::kBool) return (uint8_t)v ? 1.0f : 0.0f;
    else return static_cast<float>(v);
}

template <int OP, typename T>
struct StatReducer : Reducer<MTXC_REDUCE_SUM, T> {
    using Sum = Reducer<MTXC_REDUCE_SUM, T>;
    using State = typename Sum::State;
    static constexpr bool kVecFold = OP == kStatMean && Sum::kVecFold;  // rms / norm square each element
    static constexpr bool kColSimd = OP == kStatMean && Sum::kColSimd;
    __device__ static void fold(State& s, T v, uint32_t i) { Sum::fold(s, OP == kStatMean ? v : square_in_type(v), i); }
    // sum / (float)n in the division's dtype; *as_half tells whether that dtype is Float16
    __device__ static float mean_of(T sum, uint32_t n, bool* as_half) {
        const float nf = (float)n;
        *as_half = false;
        if constexpr (std::is_same_v<T, float>) {
            return __fdiv_rn(sum, nf);
        } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
            return to_float(from_float<T>(__fdiv_rn(to_float(sum), to_float(from_float<T>(nf)))));
        } else if constexpr (std::is_same_v<T, __half>) {
            if (n <= 65504u) {
                *as_half = true;
                return to_float(from_float<T>(__fdiv_rn(to_float(sum), to_float(from_float<T>(nf)))));
            }
            return __fdiv_rn(to_float(sum), nf);
        } else {
            return __fdiv_rn(as_float(sum), nf);
        }
    }
    __device__ static void store(const Out& o, uint64_t gid, const State& s) {
        T sum;  // the SumPrimitive's output
        if constexpr (Traits<T>::kFloat) sum = from_float<T>(s);
        else if constexpr (Traits<T>::kBool) sum = mbool(s != 0);
        else sum = (T)s;
        if constexpr (OP == kStatNorm) {
            if constexpr (std::is_same_v<T, __half> || Traits<T>::kBool)
                static_cast<__half*>(o.v)[gid] = __float2half_rn(sqrtf(as_float(sum)));
            else
                static_cast<float*>(o.v)[gid] = sqrtf(as_float(sum));
        } else {
            bool as_half;
            const float m = mean_of(sum, o.n, &as_half);
            if constexpr (OP == kStatMean) {
                if constexpr (std::is_same_v<T, __nv_bfloat16>) static_cast<T*>(o.v)[gid] = __float2bfloat16_rn(m);
                else if (as_half) static_cast<__half*>(o.v)[gid] = __float2half_rn(m);
                else static_cast<float*>(o.v)[gid] = m;
            } else {  // rms: sqrt of the mean, half only when the mean is half
                if (as_half) static_cast<__half*>(o.v)[gid] = __float2half_rn(sqrtf(m));
                else static_cast<float*>(o.v)[gid] = sqrtf(m);
            }
        }
    }
};
template <typename T>
struct Reducer<kStatMean, T> : StatReducer<kStatMean, T> {};
template <typename T>
struct Reducer<kStatRms, T> : StatReducer<kStatRms, T> {};
template <typename T>
struct Reducer<kStatNorm, T> : StatReducer<kStatNorm, T> {};

// Output dtype of a statistic (the dtype the reference's composition ends in).
int stat_out_dtype(int op, int dtype, uint32_t n) {
    switch (dtype) {
        case MTXC_FLOAT: return MTXC_FLOAT;
        case MTXC_FLOAT16: return op == kStatNorm || n <= 65504u ? MTXC_FLOAT16 : MTXC_FLOAT;
        case MTXC_BFLOAT16: return op == kStatMean ? MTXC_BFLOAT16 : MTXC_FLOAT;
        case MTXC_BOOL: return op == kStatNorm ? MTXC_FLOAT16 : MTXC_FLOAT;
        default: return MTXC_FLOAT;
    }
}

// Reducers that fold a whole vector at once (kVecFold); the others fold element by element.
template <class R, class = void>
struct VecFold : std::false_type {};
template <class R>
struct VecFold<R, std::void_t<decltype(R::kVecFold)>> : std::bool_constant<R::kVecFold> {};
// Reducers whose column kernel folds a lane's 16 bytes of columns as packed words (kColSimd).
template <class R, class = void>
struct ColSimd : std::false_type {};
template <class R>
struct ColSimd<R, std::void_t<decltype(R::kColSimd)>> : std::bool_constant<R::kColSimd> {};
// Keyed column folds (col_init_keyed: the caller supplies the carried indices' storage).
template <class R, class = void>
struct ColKeyed : std::false_type {};
template <class R>
struct ColKeyed<R, std::void_t<decltype(R::kKeyed)>> : std::bool_constant<R::kKeyed> {};
static_assert(kUnroll % 2 == 0, "col_fold_rows folds rows in pairs");

// Folds kUnroll packed rows x[k] (row numbers row0 + k * step) into a column state, two at a time where
// the reducer can.
template <class R, class X>
__device__ __forceinline__ void col_fold_rows(typename R::ColState& cs, const X (&x)[kUnroll], uint32_t row0,
                                              uint32_t step) {
    if constexpr (ColKeyed<R>::value) {  // keyed folds take two rows per call (col_fold2)
#pragma unroll
        for (int k = 0; k < kUnroll; k += 2) {
            uint32_t wa[4], wb[4];
            memcpy(wa, &x[k], 16);
            memcpy(wb, &x[k + 1], 16);
            R::col_fold2(cs, wa, wb, row0 + k * step, row0 + (k + 1) * step);
        }
    } else {
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
            uint32_t w[4];
            memcpy(w, &x[k], 16);
            R::col_fold(cs, w, row0 + k * step);
        }
    }
}

// Streams a thread's n slots (slot i at position p0 + i * step) through a packed column state in batches of
// kUnroll: the next batch's loads are issued before the current batch folds, so a warp keeps loads in flight
// while it computes, and the last partial batch is loaded at once under per-slot predicates instead of one
// slot per memory round trip.  load(x, pos) fills x from position pos.
template <class R, class X, class Load>
__device__ __forceinline__ void stream_col_fold(typename R::ColState& cs, uint32_t p0, uint32_t step, uint32_t n,
                                                Load load) {
    uint32_t i = 0;
    if (n >= (uint32_t)kUnroll) {
        X a[kUnroll], b[kUnroll];
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) load(a[k], p0 + k * step);
        while (true) {
            bool more = i + 2 * kUnroll <= n;
            if (more) {
#pragma unroll
                for (int k = 0; k < kUnroll; ++k) load(b[k], p0 + (i + kUnroll + k) * step);
            }
            col_fold_rows<R>(cs, a, p0 + i * step, step);
            i += kUnroll;
            if (!more) break;
            more = i + 2 * kUnroll <= n;
            if (more) {
#pragma unroll
                for (int k = 0; k < kUnroll; ++k) load(a[k], p0 + (i + kUnroll + k) * step);
            }
            col_fold_rows<R>(cs, b, p0 + i * step, step);
            i += kUnroll;
            if (!more) break;
        }
    }
    X t[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
        if (i + k < n) load(t[k], p0 + (i + k) * step);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
        if (i + k < n) {
            uint32_t w[4];
            memcpy(w, &t[k], 16);
            R::col_fold(cs, w, p0 + (i + k) * step);
        }
    }
}

template <typename R>
__device__ __forceinline__ void warp_reduce(typename R::State& s) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        typename R::State o = R::shfl(s, m);
        R::merge(s, o);
    }
}

// Offset of the run of output `row` (row-major over `shape`) in the input.
__device__ __forceinline__ uint64_t run_offset(uint32_t row, const Dims& d) {
    uint64_t off = 0;
#pragma unroll 1
    for (int i = (int)d.n - 1; i >= 0; --i) {
        uint32_t q, r;
        d.fdiv[i].divmod(row, q, r);
        off += (uint64_t)r * d.s1[i];
        row = q;
    }
    return off;
}

// ------------------------------------------------------------------------------------------
// rows: contiguous reduced axis
// ------------------------------------------------------------------------------------------
struct RowArgs {
    Out out;
    const void* src;
    void* partials;     // S * M states when split > 1
    uint32_t len;       // elements per run
    uint32_t seg;       // elements per split (multiple of 16 / sizeof(T) unless split == 1)
    uint32_t split;     // S
    uint32_t rows;      // M
    uint32_t chunk;     // vectors per chunk of the packed (value, index) fold
    Dims d;             // shape (with fast divisors) and input strides in s1
};

template <int OP, typename T, int G>
__global__ void __launch_bounds__(kBlock) reduce_rows_kernel(const RowArgs a) {
    using R = Reducer<OP, T>;
    using S = typename R::State;
    constexpr int V = Vec16<T>::N;
    constexpr int kUnitsPerBlock = kBlock / G;
    __shared__ S warp_partial[kBlock / 32];
    // a keyed fold's carried indices: an odd run of words per thread (lane j at word 2j, the stride of the
    // column kernel's staging slots), so a warp's accesses to one lane fall on 32 different banks
    constexpr int kCarriedRun = 2 * V + 1;
    __shared__ int32_t s_carried[ColKeyed<R>::value ? kBlock * kCarriedRun : 1];

    const int slot = threadIdx.x / G;
    const int lane = threadIdx.x % G;
    const uint64_t units = (uint64_t)a.rows * a.split;
    const T* __restrict__ src = static_cast<const T*>(a.src);

    // With G == kBlock every thread of the CTA runs the same trip count (slot == 0), so the
    // __syncthreads() of the block reduction below is reached uniformly.
    for (uint64_t u = (uint64_t)blockIdx.x * kUnitsPerBlock + slot; u < units;
         u += (uint64_t)gridDim.x * kUnitsPerBlock) {
        const uint32_t row = (uint32_t)(u / a.split);
        const uint32_t part = (uint32_t)(u - (uint64_t)row * a.split);
        const uint32_t begin = part * a.seg;
        const uint32_t end = min(a.len, begin + a.seg);
        const T* p = src + run_offset(row, a.d);

        S st[V];
#pragma unroll
        for (int j = 0; j < V; ++j) st[j] = R::init();

        // scalar head up to the first 16-byte boundary
        uint32_t head = (uint32_t)(((16u - (reinterpret_cast<uintptr_t>(p + begin) & 15u)) & 15u) / sizeof(T));
        head = min(head, end - begin);
        if ((uint32_t)lane < head) R::fold(st[0], p[begin + lane], begin + lane);
        const uint32_t vbeg = begin + head;
        const uint32_t nvec = (end - vbeg) / V;
        const T* pv = p + vbeg;
        uint32_t c = lane;
        // (value, index) of the 1- and 2-byte types but Float16: the packed fold of the column kernel,
        // its lanes being the V positions of the thread's vectors (consecutive vectors G * V elements
        // apart).  Float16 keeps the element fold, whose widening is one conversion (B200, ArgMax over
        // rows of 32,768: Float16 1.01 element-wise / 0.94 packed; BFloat16 0.86 / 0.94, int16 0.74 /
        // 0.86, int8 0.37 / 0.74 of the measured copy bandwidth)
        constexpr bool kPackedPair = !VecFold<R>::value && ColSimd<R>::value && !std::is_same_v<T, __half>;
        if constexpr (kPackedPair) {
            typename R::ColState cs = [&] {
                if constexpr (ColKeyed<R>::value) return R::col_init_keyed(G * V, a.chunk, 1, &s_carried[threadIdx.x * kCarriedRun]);
                else return R::col_init(G * V, a.chunk, 1);
            }();
            for (; c + (kUnroll - 1) * G < nvec; c += kUnroll * G) {
                Vec16<T> x[kUnroll];
#pragma unroll
                for (int k = 0; k < kUnroll; ++k) x[k] = load_stream(pv + (size_t)(c + k * G) * V);
                col_fold_rows<R>(cs, x, vbeg + c * V, G * V);
            }
            for (; c < nvec; c += G) {
                Vec16<T> x = load_stream(pv + (size_t)c * V);
                uint32_t w[4];
                memcpy(w, &x, 16);
                R::col_fold(cs, w, vbeg + c * V);
            }
            S lanes[V];
            R::col_finish(cs, lanes);
#pragma unroll
            for (int j = 0; j < V; ++j) R::merge(st[j], lanes[j]);
        }
        [[maybe_unused]] Lanes pk;
        if constexpr (VecFold<R>::value) pk = R::vec_init();
        if constexpr (!kPackedPair)
        for (; c + (kUnroll - 1) * G < nvec; c += kUnroll * G) {
            Vec16<T> x[kUnroll];
#pragma unroll
            for (int k = 0; k < kUnroll; ++k) x[k] = load_stream(pv + (size_t)(c + k * G) * V);
#pragma unroll
            for (int k = 0; k < kUnroll; ++k) {
                if constexpr (VecFold<R>::value) {
                    R::vec_fold(pk, x[k]);
                } else {
#pragma unroll
                    for (int j = 0; j < V; ++j) R::fold(st[j], x[k].v[j], vbeg + (c + k * G) * V + j);
                }
            }
        }
        if constexpr (!kPackedPair)
        for (; c < nvec; c += G) {
            Vec16<T> x = load_stream(pv + (size_t)c * V);
            if constexpr (VecFold<R>::value) {
                R::vec_fold(pk, x);
            } else {
#pragma unroll
                for (int j = 0; j < V; ++j) R::fold(st[j], x.v[j], vbeg + c * V + j);
            }
        }
        if constexpr (VecFold<R>::value) R::vec_finish(st[0], pk);
        for (uint32_t i = vbeg + nvec * V + lane; i < end; i += G) R::fold(st[0], p[i], i);

#pragma unroll
        for (int j = 1; j < V; ++j) R::merge(st[0], st[j]);
        warp_reduce<R>(st[0]);
        if constexpr (G == kBlock) {
            if ((threadIdx.x & 31) == 0) warp_partial[threadIdx.x / 32] = st[0];
            __syncthreads();
            if (threadIdx.x < 32) {
                // init() is an identity for every reducer: a (value, index) state still equal
                // to its initial value was never updated, so its index is 0, as init's is.
                S s = threadIdx.x < kBlock / 32 ? warp_partial[threadIdx.x] : R::init();
                warp_reduce<R>(s);
                st[0] = s;
            }
            __syncthreads();
        }
        if (lane == 0) {
            if (a.split == 1) R::store(a.out, row, st[0]);
            else static_cast<S*>(a.partials)[(uint64_t)part * a.rows + row] = st[0];
        }
    }
}

// ------------------------------------------------------------------------------------------
// cols: strided reduced axis, contiguous innermost output axis
// ------------------------------------------------------------------------------------------
struct ColArgs {
    Out out;
    const void* src;
    void* partials;
    uint32_t len;         // reduced axis length
    uint32_t rstride;     // reduced axis stride (elements)
    uint32_t seg;         // reduced rows per split
    uint32_t split;
    uint32_t inner;       // extent of the innermost output axis
    uint32_t outer;       // product of the other output axes
    uint32_t col_tiles;   // CTAs across `inner`
    uint32_t tx;          // threads across columns (power of two, <= 32)
    uint64_t outputs;     // M = outer * inner
    uint32_t chunk;       // rows per chunk of the packed (value, index) column fold
    Dims d;               // outer axes: shape (fast divisors) and input strides in s1
};

// Rows (or row vectors) per chunk of the packed (value, index) fold: 65,535 (the 16-bit chunk numbers' range).  A lower value
// changes no result, only how often the chunk numbers turn into row indices; it is settable so tests can
// reach that step at small sizes (mtxc_debug_set_col_chunk, not part of the public header).
std::atomic<uint32_t> g_col_chunk{65535};

template <int OP, typename T, int V>
__global__ void __launch_bounds__(kBlock) reduce_cols_kernel(const ColArgs a) {
    using R = Reducer<OP, T>;
    using S = typename R::State;
    // each thread's V states, padded by one so that a warp's stores (one state each, threads VP states
    // apart) spread over the banks instead of landing V states apart on the same ones
    constexpr int VP = V + 1;
    __shared__ S partial[kBlock * VP];

    const uint32_t tx = threadIdx.x % a.tx;
    const uint32_t ty = threadIdx.x / a.tx;
    const uint32_t ty_count = kBlock / a.tx;
    uint32_t b = blockIdx.x;
    const uint32_t tile = b % a.col_tiles;
    b /= a.col_tiles;
    const uint32_t o = b % a.outer;
    const uint32_t part = b / a.outer;
    const uint32_t col = (tile * a.tx + tx) * V;
    const bool active = col < a.inner;

    S st[V];
#pragma unroll
    for (int j = 0; j < V; ++j) st[j] = R::init();

    if (active) {
        const T* __restrict__ p = static_cast<const T*>(a.src) + run_offset(o, a.d) + col;
        const uint32_t begin = part * a.seg;
        const uint32_t end = min(a.len, begin + a.seg);
        uint32_t r = begin + ty;
        const uint32_t step = ty_count;
        if constexpr (ColSimd<R>::value && V * sizeof(T) == 16) {
            // a keyed fold keeps its carried indices in this thread's staging slots (free until the epilogue)
            typename R::ColState cs = [&] {
                if constexpr (ColKeyed<R>::value)
                    return R::col_init_keyed(step, a.chunk, 0, &partial[threadIdx.x * VP].i);
                else return R::col_init(step, a.chunk);
            }();
            // the packed folds stream (next rows' loads in flight while the current ones fold: uint16 ArgMax
            // 0.83 -> 0.90 of the copy figure on B200), except the 1-byte keyed fold, whose 16 keys plus a second
            // batch of loads cost a CTA per SM before its indices moved to shared memory and gain nothing since
            if constexpr (!(ColKeyed<R>::value && sizeof(T) == 1)) {
                const uint32_t n = r < end ? (end - 1 - r) / step + 1 : 0;
                const uint32_t rs = a.rstride;
                stream_col_fold<R, ew::Slot<T, V>>(cs, r, step, n, [&](ew::Slot<T, V>& x, uint32_t row) {
                    ew::load_slot(x, p + (size_t)row * rs);
                });
            } else {
                for (; r + (kUnroll - 1) * step < end; r += kUnroll * step) {
                    ew::Slot<T, V> x[kUnroll];
#pragma unroll
                    for (int k = 0; k < kUnroll; ++k) ew::load_slot(x[k], p + (size_t)(r + k * step) * a.rstride);
                    col_fold_rows<R>(cs, x, r, step);
                }
                for (; r < end; r += step) {
                    ew::Slot<T, V> x;
                    ew::load_slot(x, p + (size_t)r * a.rstride);
                    uint32_t w[4];
                    memcpy(w, &x, 16);
                    R::col_fold(cs, w, r);
                }
            }
            R::col_finish(cs, st);
        } else if constexpr (V > 1) {
            for (; r + (kUnroll - 1) * step < end; r += kUnroll * step) {
                ew::Slot<T, V> x[kUnroll];
#pragma unroll
                for (int k = 0; k < kUnroll; ++k) ew::load_slot(x[k], p + (size_t)(r + k * step) * a.rstride);
#pragma unroll
                for (int k = 0; k < kUnroll; ++k)
#pragma unroll
                    for (int j = 0; j < V; ++j) R::fold(st[j], x[k].v[j], r + k * step);
            }
            for (; r < end; r += step) {
                ew::Slot<T, V> x;
                ew::load_slot(x, p + (size_t)r * a.rstride);
#pragma unroll
                for (int j = 0; j < V; ++j) R::fold(st[j], x.v[j], r);
            }
        } else {
            for (; r + (kUnroll - 1) * step < end; r += kUnroll * step) {
                T x[kUnroll];
#pragma unroll
                for (int k = 0; k < kUnroll; ++k) x[k] = load_scalar_stream(p + (size_t)(r + k * step) * a.rstride);
#pragma unroll
                for (int k = 0; k < kUnroll; ++k) R::fold(st[0], x[k], r + k * step);
            }
            for (; r < end; r += step) R::fold(st[0], load_scalar_stream(p + (size_t)r * a.rstride), r);
        }
    }
#pragma unroll
    for (int j = 0; j < V; ++j) partial[threadIdx.x * VP + j] = st[j];
    __syncthreads();
    if constexpr (IsPair<S>::value) {
        // (value, index) states: the tile's tx * V outputs are finished by all threads, consecutive
        // outputs on consecutive threads (coalesced stores).  Output q (lane x = q / V, element j = q % V)
        // sits at partial[(t * tx + x) * VP + j] for row group t and merges them in ascending t, the order of
        // the single-thread merge below (B200, ArgMax over axis 1 of [16f, 8192, 1024]: int8 0.45 ->
        // 0.60, int16 0.71 -> 0.76, Float16 0.87 -> 0.91 of the measured copy bandwidth; for value
        // states, whose merges are cheap, one warp finishing alone measured faster)
        const uint32_t tile_outputs = a.tx * V;
        const uint32_t tile_col = tile * tile_outputs;
        const uint64_t gbase = (uint64_t)o * a.inner + tile_col;
        for (uint32_t q = threadIdx.x; q < tile_outputs && tile_col + q < a.inner; q += kBlock) {
            const uint32_t x = q / V, j = q % V;
            S s = partial[x * VP + j];
            for (uint32_t t = 1; t < ty_count; ++t) R::merge(s, partial[(t * a.tx + x) * VP + j]);
            if (a.split == 1) R::store(a.out, gbase + q, s);
            else static_cast<S*>(a.partials)[(uint64_t)part * a.outputs + gbase + q] = s;
        }
    } else if (ty == 0 && active) {
        for (uint32_t t = 1; t < ty_count; ++t) {
#pragma unroll
            for (int j = 0; j < V; ++j) R::merge(st[j], partial[(t * a.tx + tx) * VP + j]);
        }
        const uint64_t gid = (uint64_t)o * a.inner + col;
#pragma unroll
        for (int j = 0; j < V; ++j) {
            if (a.split == 1) R::store(a.out, gid + j, st[j]);
            else static_cast<S*>(a.partials)[(uint64_t)part * a.outputs + gid + j] = st[j];
        }
    }
}

// ------------------------------------------------------------------------------------------
// finalize: merge split partials in a fixed order
// ------------------------------------------------------------------------------------------
template <int OP, typename T>
__global__ void __launch_bounds__(kBlock) reduce_finalize_kernel(const Out dst, const void* partials, uint64_t outputs,
                                                                 uint32_t split) {
    using R = Reducer<OP, T>;
    using S = typename R::State;
    const S* ps = static_cast<const S*>(partials);
    for (uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < outputs;
         gid += (uint64_t)gridDim.x * blockDim.x) {
        S s = ps[gid];
        for (uint32_t k = 1; k < split; ++k) R::merge(s, ps[(uint64_t)k * outputs + gid]);
        R::store(dst, gid, s);
    }
}

// The same merge with one warp per output, for many splits: lane l merges partials l, l + 32, ... in
// order, then the warp combines its lanes in a fixed shuffle tree (deterministic for a given split;
// init() is the identity of every merge).
template <int OP, typename T>
__global__ void __launch_bounds__(kBlock) reduce_finalize_warp_kernel(const Out dst, const void* partials,
                                                                      uint64_t outputs, uint32_t split) {
    using R = Reducer<OP, T>;
    using S = typename R::State;
    const S* ps = static_cast<const S*>(partials);
    const uint32_t lane = threadIdx.x % 32;
    const uint64_t warps = (uint64_t)gridDim.x * (kBlock / 32);
    for (uint64_t gid = (uint64_t)blockIdx.x * (kBlock / 32) + threadIdx.x / 32; gid < outputs; gid += warps) {
        S s = R::init();
        for (uint32_t k = lane; k < split; k += 32) R::merge(s, ps[(uint64_t)k * outputs + gid]);
        warp_reduce<R>(s);
        if (lane == 0) R::store(dst, gid, s);
    }
}

// ------------------------------------------------------------------------------------------
// generic: one thread per output, the reference CPU loop (Matrix.mm:15193-15205)
// ------------------------------------------------------------------------------------------
struct GenericArgs {
    Out out;
    const void* src;
    uint64_t outputs;
    uint32_t len;
    uint32_t rstride;
    uint32_t cdims;
    uint32_t s_out[MTXC_MAX_DIMS];
    uint32_t s_in[MTXC_MAX_DIMS];
};

template <int OP, typename T>
__global__ void __launch_bounds__(kBlock) reduce_generic_kernel(const GenericArgs a) {
    using R = Reducer<OP, T>;
    const T* __restrict__ src = static_cast<const T*>(a.src);
    for (uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < a.outputs;
         gid += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t off = 0, rem = gid;
        for (uint32_t i = 0; i < a.cdims; ++i) {
            off += (rem / a.s_out[i]) * a.s_in[i];
            rem %= a.s_out[i];
        }
        typename R::State s = R::init();
        const T* p = src + off;
        for (uint32_t i = 0; i < a.len; ++i) R::fold(s, p[(uint64_t)i * a.rstride], i);
        R::store(a.out, gid, s);
    }
}

// ------------------------------------------------------------------------------------------
// host planning
// ------------------------------------------------------------------------------------------
int blocks_per_sm(const void* kernel) {
    static std::mutex mu;
    static std::map<const void*, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(kernel);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kBlock, 0) != cudaSuccess || n < 1) n = 1;
    cache[kernel] = n;
    return n;
}

// Picks the split count in [1, max_split] whose CTA count fills whole waves best, preferring
// at least one full wave and then fewer splits.
uint32_t choose_split(uint64_t base_units, uint64_t units_per_wave, uint32_t max_split) {
    if (base_units >= units_per_wave || max_split <= 1) return 1;
    uint32_t best = 1;
    double best_score = -1.0;
    for (uint32_t s = 1; s <= max_split; ++s) {
        const uint64_t units = base_units * s;
        const uint64_t waves = (units + units_per_wave - 1) / units_per_wave;
        double eff = (double)units / (double)(waves * units_per_wave);
        if (units < units_per_wave) eff *= 0.5;  // under one wave: idle SMs
        if (eff > best_score + 1e-9) {
            best_score = eff;
            best = s;
        }
        if (units >= 4 * units_per_wave) break;
    }
    return best;
}

enum class Plan { kRows, kCols, kGeneric };

struct ReducePlan {
    Plan kind = Plan::kGeneric;
    int group = 32;       // rows: threads per unit
    int vec = 1;          // cols: elements per thread
    uint32_t split = 1;
    uint32_t seg = 0;
    uint32_t tx = 32;
    uint64_t outputs = 0;
    size_t partial_bytes = 0;
};

struct Meta {
    uint32_t cdims;
    uint32_t shape[MTXC_MAX_DIMS];
    uint32_t s_out[MTXC_MAX_DIMS];
    uint32_t s_in[MTXC_MAX_DIMS];
};

template <int OP, typename T>
ReducePlan plan_reduce(const Meta& m, const void* src, uint32_t rstride, uint32_t len, size_t workspace_bytes,
                       int sm_count) {
    using S = typename Reducer<OP, T>::State;
    constexpr uint32_t V = Vec16<T>::N;
    ReducePlan p;
    p.outputs = product(m.shape, m.cdims);
    if (p.outputs == 0 || len == 0 || p.outputs >= (1ull << 32) || !is_row_major(m.shape, m.s_out, m.cdims))
        return p;
    const uint32_t k = m.cdims - 1;
    const uint64_t max_partials = workspace_bytes / sizeof(S);
    if (rstride == 1 && len >= 32) {
        p.kind = Plan::kRows;
        const uint64_t warp_slots = (uint64_t)sm_count * 64;
        uint32_t max_split;
        if (len <= 32 * V * 8 || p.outputs >= warp_slots) {
            p.group = 32;
            max_split = std::max<uint32_t>(1, len / (32 * V * kUnroll));
            p.split = choose_split(p.outputs, warp_slots, max_split);
        } else {
            p.group = kBlock;
            const void* fn = (const void*)reduce_rows_kernel<OP, T, kBlock>;
            const uint64_t block_slots = (uint64_t)sm_count * blocks_per_sm(fn);
            max_split = std::max<uint32_t>(1, len / (kBlock * V * kUnroll));
            p.split = choose_split(p.outputs, block_slots, max_split);
        }
        // a split axis streams best as about four waves of shorter segments rather than one wave of
        // long ones (B200, 16 GiB full sum: 0.92 -> 1.11 of the measured copy bandwidth)
        if (p.split > 1) p.split = (uint32_t)std::min<uint64_t>((uint64_t)p.split * kSplitWaves, max_split);
        while (p.split > 1 && p.outputs * p.split > max_partials) p.split /= 2;
        p.seg = p.split == 1 ? len : (uint32_t)(((uint64_t)len + p.split - 1) / p.split + V - 1) / V * V;
        if (p.split > 1) p.split = (len + p.seg - 1) / p.seg;
        p.partial_bytes = p.split > 1 ? p.outputs * p.split * sizeof(S) : 0;
        return p;
    }
    if (rstride != 1 && m.s_in[k] == 1 && m.shape[k] >= 2) {
        p.kind = Plan::kCols;
        constexpr uint32_t VC = col_vec<OP, T>();
        constexpr uint32_t VN = col_vec_narrow<T>();
        const uint32_t inner = m.shape[k];
        auto vec_ok = [&](uint32_t vc) {
            bool ok = reinterpret_cast<uintptr_t>(src) % (vc * sizeof(T)) == 0 && inner % vc == 0 && rstride % vc == 0;
            for (uint32_t i = 0; i < k; ++i) ok = ok && (m.shape[i] == 1 || m.s_in[i] % vc == 0);
            return ok;
        };
        p.vec = vec_ok(VC) ? (int)VC : VN > 1 && vec_ok(VN) ? (int)VN : 1;
        const uint32_t threads_across = (inner + p.vec - 1) / p.vec;
        uint32_t tx = 1;
        while (tx < threads_across && tx < 32) tx <<= 1;
        p.tx = tx;
        const uint64_t col_tiles = (threads_across + tx - 1) / tx;
        const uint64_t base = col_tiles * (p.outputs / inner);
        // the split is planned with the vector kernel's occupancy whatever the alignment, so
        // the workspace a call needs does not depend on its pointers
        const void* fn = (const void*)reduce_cols_kernel<OP, T, VC>;
        const uint64_t block_slots = (uint64_t)sm_count * blocks_per_sm(fn);
        const uint32_t ty_count = kBlock / tx;
        const uint32_t max_split = std::max<uint32_t>(1, len / (ty_count * 8));
        p.split = choose_split(base, block_slots, max_split);
        while (p.split > 1 && p.outputs * p.split > max_partials) p.split /= 2;
        p.seg = (len + p.split - 1) / p.split;
        p.split = (len + p.seg - 1) / p.seg;
        p.partial_bytes = p.split > 1 ? p.outputs * p.split * sizeof(S) : 0;
        return p;
    }
    return p;
}

template <int OP, typename T>
int launch_reduce(const Meta& m, const Out dst, const void* src, uint32_t rstride, uint32_t len, void* workspace,
                  size_t workspace_bytes, int sm_count, cudaStream_t stream) {
    const ReducePlan p = plan_reduce<OP, T>(m, src, rstride, len, workspace_bytes, sm_count);
    if (p.outputs == 0) return MTXC_OK;
    if (p.partial_bytes > workspace_bytes)
        return fail(MTXC_ERR_WORKSPACE, "mtxc_reduce: workspace too small for the split partials");
    const uint32_t k = m.cdims - 1;
    if (p.kind == Plan::kRows) {
        RowArgs a{};
        a.out = dst;
        a.src = src;
        a.partials = workspace;
        a.len = len;
        a.seg = p.seg;
        a.split = p.split;
        a.rows = (uint32_t)p.outputs;
        a.chunk = g_col_chunk.load(std::memory_order_relaxed);
        a.d.n = m.cdims;
        for (uint32_t i = 0; i < m.cdims; ++i) {
            a.d.shape[i] = m.shape[i];
            a.d.s1[i] = m.s_in[i];
            a.d.fdiv[i] = FastDiv(m.shape[i]);
        }
        const uint64_t units = p.outputs * p.split;
        const uint64_t upb = kBlock / p.group;
        uint64_t blocks = (units + upb - 1) / upb;
        blocks = std::min<uint64_t>(blocks, (uint64_t)sm_count * 64);
        if (p.group == 32) reduce_rows_kernel<OP, T, 32><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        else reduce_rows_kernel<OP, T, kBlock><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        if (int rc = check_launch("reduce_rows_kernel")) return rc;
    } else if (p.kind == Plan::kCols) {
        ColArgs a{};
        a.out = dst;
        a.src = src;
        a.partials = workspace;
        a.len = len;
        a.rstride = rstride;
        a.seg = p.seg;
        a.split = p.split;
        a.inner = m.shape[k];
        a.outer = (uint32_t)(p.outputs / m.shape[k]);
        a.tx = p.tx;
        a.col_tiles = (((a.inner + p.vec - 1) / p.vec) + p.tx - 1) / p.tx;
        a.outputs = p.outputs;
        a.chunk = g_col_chunk.load(std::memory_order_relaxed);
        a.d.n = k;
        for (uint32_t i = 0; i < k; ++i) {
            a.d.shape[i] = m.shape[i];
            a.d.s1[i] = m.s_in[i];
            a.d.fdiv[i] = FastDiv(m.shape[i]);
        }
        const uint64_t blocks = (uint64_t)a.col_tiles * a.outer * p.split;
        if (blocks >= (1ull << 31)) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: too many column tiles");
        constexpr int VN = col_vec_narrow<T>();
        if (p.vec == col_vec<OP, T>()) reduce_cols_kernel<OP, T, col_vec<OP, T>()><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        else if (VN > 1 && p.vec == VN) reduce_cols_kernel<OP, T, VN><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        else reduce_cols_kernel<OP, T, 1><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        if (int rc = check_launch("reduce_cols_kernel")) return rc;
    } else {
        GenericArgs a{};
        a.out = dst;
        a.src = src;
        a.outputs = p.outputs;
        a.len = len;
        a.rstride = rstride;
        a.cdims = m.cdims;
        for (uint32_t i = 0; i < m.cdims; ++i) {
            a.s_out[i] = m.s_out[i];
            a.s_in[i] = m.s_in[i];
        }
        const uint64_t blocks = std::min<uint64_t>((p.outputs + kBlock - 1) / kBlock, (uint64_t)sm_count * 32);
        reduce_generic_kernel<OP, T><<<(unsigned)blocks, kBlock, 0, stream>>>(a);
        return check_launch("reduce_generic_kernel");
    }
    if (p.split >= 32) {
        const uint64_t blocks = std::min<uint64_t>((p.outputs + kBlock / 32 - 1) / (kBlock / 32), (uint64_t)sm_count * 32);
        reduce_finalize_warp_kernel<OP, T><<<(unsigned)blocks, kBlock, 0, stream>>>(dst, workspace, p.outputs, p.split);
        if (int rc = check_launch("reduce_finalize_warp_kernel")) return rc;
    } else if (p.split > 1) {
        const uint64_t blocks = std::min<uint64_t>((p.outputs + kBlock - 1) / kBlock, (uint64_t)sm_count * 32);
        reduce_finalize_kernel<OP, T><<<(unsigned)blocks, kBlock, 0, stream>>>(dst, workspace, p.outputs, p.split);
        if (int rc = check_launch("reduce_finalize_kernel")) return rc;
    }
    return MTXC_OK;
}

template <typename T>
int launch_reduce_op(int op, const Meta& m, const Out dst, const void* src, uint32_t rstride, uint32_t len, void* ws,
                     size_t wsb, int sms, cudaStream_t st) {
    switch (op) {
        case MTXC_REDUCE_SUM: return launch_reduce<MTXC_REDUCE_SUM, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case MTXC_REDUCE_MAX: return launch_reduce<MTXC_REDUCE_MAX, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case MTXC_REDUCE_MIN: return launch_reduce<MTXC_REDUCE_MIN, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case MTXC_REDUCE_ARGMAX: return launch_reduce<MTXC_REDUCE_ARGMAX, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case MTXC_REDUCE_ARGMIN: return launch_reduce<MTXC_REDUCE_ARGMIN, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case kPairMax: return launch_reduce<kPairMax, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case kPairMin: return launch_reduce<kPairMin, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case kStatMean: return launch_reduce<kStatMean, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case kStatRms: return launch_reduce<kStatRms, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        case kStatNorm: return launch_reduce<kStatNorm, T>(m, dst, src, rstride, len, ws, wsb, sms, st);
        default: return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: unknown op");
    }
}

template <typename T>
size_t partial_bytes_op(int op, const Meta& m, const void* src, uint32_t rstride, uint32_t len, int sms) {
    const size_t unlimited = ~size_t(0) / 2;
    switch (op) {
        case MTXC_REDUCE_SUM: return plan_reduce<MTXC_REDUCE_SUM, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        case MTXC_REDUCE_MAX: return plan_reduce<MTXC_REDUCE_MAX, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        case MTXC_REDUCE_MIN: return plan_reduce<MTXC_REDUCE_MIN, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        case MTXC_REDUCE_ARGMAX: return plan_reduce<MTXC_REDUCE_ARGMAX, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        case kPairMax: return plan_reduce<kPairMax, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        case kPairMin: return plan_reduce<kPairMin, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        case kStatMean:
        case kStatRms:
        case kStatNorm: return plan_reduce<MTXC_REDUCE_SUM, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
        default: return plan_reduce<MTXC_REDUCE_ARGMIN, T>(m, src, rstride, len, unlimited, sms).partial_bytes;
    }
}

int make_meta(uint32_t cdims, const uint32_t* shape, const uint32_t* s_out, const uint32_t* s_in, Meta& m) {
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: cdims > MTXC_MAX_DIMS");
    if (cdims == 0) {
        // the reference's single-output case (Matrix.mm:15121-15126)
        m.cdims = 1;
        m.shape[0] = 1;
        m.s_out[0] = 1;
        m.s_in[0] = 1;
        return MTXC_OK;
    }
    if (!shape || !s_out || !s_in) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: null metadata pointer");
    m.cdims = cdims;
    for (uint32_t i = 0; i < cdims; ++i) {
        if (s_out[i] == 0 && shape[i] > 1)
            return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: zero output stride");
        m.shape[i] = shape[i];
        m.s_out[i] = s_out[i] ? s_out[i] : 1;
        m.s_in[i] = s_in[i];
    }
    return MTXC_OK;
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_reduce(int op, int dtype, void* dst, const void* src, uint32_t reduce_stride, uint32_t reduce_len,
                           uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides,
                           const uint32_t* src_strides) {
    if (int rc = require_init()) return rc;
    if (op < MTXC_REDUCE_SUM || op > MTXC_REDUCE_ARGMIN) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: unknown op");
    Meta m;
    if (int rc = make_meta(cdims, shape, dst_strides, src_strides, m)) return rc;
    if (product(m.shape, m.cdims) == 0) return MTXC_OK;
    if (!dst || (!src && reduce_len)) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce: null buffer");
    ThreadCtx& c = ctx();
    int rc = MTXC_OK;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_reduce_op<T>(op, m, Out{dst, nullptr}, src, reduce_stride, reduce_len, c.workspace, c.workspace_bytes, c.sm_count,
                                 c.stream());
    });
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_reduce: no kernel for dtype ") + dtype_name(dtype));
    return rc;
}

extern "C" int mtxc_reduce_stat_dtype(int stat, int dtype, uint32_t reduce_len) {
    if (stat < MTXC_STAT_MEAN || stat > MTXC_STAT_NORM) return -1;
    if (!dispatch_dtype(dtype, [](auto*) {})) return -1;
    return stat_out_dtype(kStatMean + stat, dtype, reduce_len);
}

extern "C" int mtxc_reduce_stat(int stat, int dtype, void* dst, const void* src, uint32_t reduce_stride,
                                uint32_t reduce_len, uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides,
                                const uint32_t* src_strides) {
    if (int rc = require_init()) return rc;
    if (stat < MTXC_STAT_MEAN || stat > MTXC_STAT_NORM)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_stat: unknown statistic");
    Meta m;
    if (int rc = make_meta(cdims, shape, dst_strides, src_strides, m)) return rc;
    if (!dispatch_dtype(dtype, [](auto*) {}))
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_reduce_stat: no kernel for dtype ") + dtype_name(dtype));
    if (product(m.shape, m.cdims) == 0) return MTXC_OK;
    if (!dst || (!src && reduce_len)) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_stat: null buffer");
    ThreadCtx& c = ctx();
    int rc = MTXC_OK;
    Out out{dst, nullptr};
    out.n = reduce_len;
    dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_reduce_op<T>(kStatMean + stat, m, out, src, reduce_stride, reduce_len, c.workspace,
                                 c.workspace_bytes, c.sm_count, c.stream());
    });
    return rc;
}

extern "C" int mtxc_reduce_workspace_bytes(int op, int dtype, uint32_t reduce_stride, uint32_t reduce_len,
                                           uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides,
                                           const uint32_t* src_strides, size_t* bytes) {
    if (!bytes) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_workspace_bytes: null pointer");
    if (op < MTXC_REDUCE_SUM || op > MTXC_REDUCE_ARGMIN)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_workspace_bytes: unknown op");
    Meta m;
    if (int rc = make_meta(cdims, shape, dst_strides, src_strides, m)) return rc;
    const int sms = ctx().device >= 0 ? ctx().sm_count : 148;
    size_t b = 0;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        // alignment only affects the column kernel's vector width, not the partial count
        b = partial_bytes_op<T>(op, m, nullptr, reduce_stride, reduce_len, sms);
    });
    if (!known) return fail(MTXC_ERR_UNSUPPORTED_DTYPE, "mtxc_reduce_workspace_bytes: unsupported dtype");
    *bytes = b;
    return MTXC_OK;
}

// ------------------------------------------------------------------------------------------
// mtxc_reduce_noalloc: mtxc_reduce with its split partials in a static device array, for callers
// that cannot allocate device memory.
// ------------------------------------------------------------------------------------------

// The scratch itself.  It is part of this library's device image: every GPU that loads the library
// holds it until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MTXC_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxNoallocDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_address[kMaxNoallocDevices] = {};
// The size the refusal check compares against: the array's size, lowered only by the test hook
// mtxc_debug_set_noalloc_limit (not in the public header) so tests can reach the refusal at small sizes.
std::atomic<size_t> g_noalloc_limit{MTXC_NOALLOC_SCRATCH_BYTES};

// In host code `g_noalloc_scratch` is only a host-side stand-in for the array; handing it to a kernel
// would fault (or, where the GPU can reach host memory, silently use the wrong memory).  Its device
// address is looked up once per device, with that device current, and cached.
int noalloc_scratch_address(int device, void** out) {
    if (device < 0 || device >= kMaxNoallocDevices)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_address[device]) {
        int current = -1;
        cudaError_t err = cudaGetDevice(&current);
        if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
        if (current != device && (err = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (current != device) cudaSetDevice(current);
        if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(noalloc scratch)");
        g_noalloc_address[device] = p;
    }
    *out = g_noalloc_address[device];
    return MTXC_OK;
}

}  // namespace

// Forgets the cached scratch address of `device` (mtxc_shutdown): a device reset behind the library
// reloads its device image, so the next first call looks the address up again.
void mtxc::noalloc_forget(int device) {
    if (device < 0 || device >= kMaxNoallocDevices) return;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    g_noalloc_address[device] = nullptr;
}

extern "C" int mtxc_reduce_noalloc(int op, int dtype, void* dst, const void* src, uint32_t reduce_stride,
                                   uint32_t reduce_len, uint32_t cdims, const uint32_t* shape,
                                   const uint32_t* dst_strides, const uint32_t* src_strides) {
    if (int rc = require_init()) return rc;
    if (op < MTXC_REDUCE_SUM || op > MTXC_REDUCE_ARGMIN)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_noalloc: unknown op");
    Meta m;
    if (int rc = make_meta(cdims, shape, dst_strides, src_strides, m)) return rc;
    if (product(m.shape, m.cdims) == 0) return MTXC_OK;
    if (!dst || (!src && reduce_len)) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_noalloc: null buffer");
    ThreadCtx& c = ctx();
    size_t need = 0;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        need = partial_bytes_op<T>(op, m, src, reduce_stride, reduce_len, c.sm_count);
    });
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE,
                    std::string("mtxc_reduce_noalloc: no kernel for dtype ") + dtype_name(dtype));
    const size_t limit = g_noalloc_limit.load(std::memory_order_relaxed);
    if (need > limit)
        return fail(MTXC_ERR_WORKSPACE, "mtxc_reduce_noalloc: this reduction splits into " + std::to_string(need) +
                                            " bytes of partials, more than the " + std::to_string(limit) +
                                            "-byte static scratch; use mtxc_reduce with a workspace");
    void* scratch = nullptr;
    if (need) {
        if (int rc = noalloc_scratch_address(c.device, &scratch)) return rc;
    }
    int rc = MTXC_OK;
    dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_reduce_op<T>(op, m, Out{dst, nullptr}, src, reduce_stride, reduce_len, scratch,
                                 scratch ? (size_t)MTXC_NOALLOC_SCRATCH_BYTES : 0, c.sm_count, c.stream());
    });
    return rc;
}

// ------------------------------------------------------------------------------------------
// mtxc_reduce_pair: Max and ArgMax (Min and ArgMin) from one read of the input.
// ------------------------------------------------------------------------------------------
extern "C" int mtxc_reduce_pair(int op, int dtype, void* dst_values, int32_t* dst_indices, const void* src,
                                uint32_t reduce_stride, uint32_t reduce_len, uint32_t cdims, const uint32_t* shape,
                                const uint32_t* dst_strides, const uint32_t* src_strides) {
    if (int rc = require_init()) return rc;
    int pair_op;
    if (op == MTXC_REDUCE_MAX || op == MTXC_REDUCE_ARGMAX) pair_op = kPairMax;
    else if (op == MTXC_REDUCE_MIN || op == MTXC_REDUCE_ARGMIN) pair_op = kPairMin;
    else return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_pair: op must be MAX / ARGMAX or MIN / ARGMIN");
    Meta m;
    if (int rc = make_meta(cdims, shape, dst_strides, src_strides, m)) return rc;
    if (product(m.shape, m.cdims) == 0) return MTXC_OK;
    if (!dst_values || !dst_indices || (!src && reduce_len))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_pair: null buffer");
    ThreadCtx& c = ctx();
    int rc = MTXC_OK;
    const bool known = dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_reduce_op<T>(pair_op, m, Out{dst_values, dst_indices}, src, reduce_stride, reduce_len, c.workspace,
                                 c.workspace_bytes, c.sm_count, c.stream());
    });
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_reduce_pair: no kernel for dtype ") + dtype_name(dtype));
    return rc;
}

// Test hook: the size mtxc_reduce_noalloc's refusal compares against (clamped to the array's size; 0 restores
// it); returns the previous value.  The array itself keeps its size.
extern "C" size_t mtxc_debug_set_noalloc_limit(size_t bytes) {
    const size_t v = bytes == 0 || bytes > MTXC_NOALLOC_SCRATCH_BYTES ? (size_t)MTXC_NOALLOC_SCRATCH_BYTES : bytes;
    return g_noalloc_limit.exchange(v);
}

// Test hook: rows per chunk of the packed column fold (clamped to 1 .. 65,535); returns the previous value.
extern "C" uint32_t mtxc_debug_set_col_chunk(uint32_t rows) {
    const uint32_t v = rows < 1 ? 1 : rows > 65535 ? 65535 : rows;
    return mtxc::g_col_chunk.exchange(v);
}
