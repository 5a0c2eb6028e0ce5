// Tests of the C++ host mirror (matrix_b200/host/mtx.hpp) on a GPU, written the way a user of the
// reference writes matrix code: build lazy expressions, eval() / compile() / execute() them, read
// the results back.  Expected values come from the CPU oracle (oracle/liboracle.so), which restates
// the reference's CPU eval; comparison rules as in tests/helpers.py (bit-exact, all NaNs equal;
// float sums within 1e-5 * sum|x|; exp within 2 ulp; softmax within a relative 1e-5).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "mtx.hpp"

extern "C" {
uint32_t orc_collapse3(const uint32_t*, const uint32_t*, const uint32_t*, const uint32_t*, uint32_t, uint64_t, uint32_t*,
                       uint32_t*, uint32_t*, uint32_t*);
uint32_t orc_collapse_reduce2(const uint32_t*, const uint32_t*, const uint32_t*, uint32_t, int, int, int, uint64_t,
                              uint32_t*, uint32_t*, uint32_t*);
int orc_broadcast_shapes(const uint32_t*, const uint32_t*, int, const uint32_t*, const uint32_t*, int, uint32_t*,
                         uint32_t*, uint32_t*, uint32_t*, uint32_t*, uint32_t*);
int orc_reduce(int, int, void*, const void*, uint32_t, uint32_t, uint32_t, const uint32_t*, const uint32_t*,
               const uint32_t*, uint64_t, int);
int orc_broadcast(int, int, void*, const void*, const void*, uint32_t, const uint32_t*, const uint32_t*, const uint32_t*,
                  uint64_t, int);
int orc_arange(int, void*, const void*, const void*, uint64_t);
int orc_sum_flat(int, void*, const void*, uint64_t);
}

using mtx::dtype;
using mtx::matrix;
using mtx::size_m;

static int checks = 0, failures = 0;

#define EXPECT(cond, ...)                          \
    do {                                           \
        ++checks;                                  \
        if (!(cond)) {                             \
            ++failures;                            \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);              \
            std::printf("\n");                     \
        }                                          \
    } while (0)

static std::vector<size_m> row_major(const std::vector<size_m>& shape) {
    std::vector<size_m> s(shape.size());
    size_m acc = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
        s[i] = acc;
        acc *= shape[i];
    }
    return s;
}

static uint64_t total(const std::vector<size_m>& s) {
    uint64_t p = 1;
    for (auto e : s) p *= e;
    return p;
}

// Oracle: x.op(axis, keepdims) on host data with the given view strides
template <typename T>
static std::vector<uint8_t> oracle_reduce(int op, const std::vector<T>& base, const std::vector<size_m>& shape,
                                          const std::vector<size_m>& strides, int axis, bool keep, int dtype_code) {
    const uint32_t dims = (uint32_t)shape.size();
    std::vector<size_m> out_shape = shape;
    if (keep) out_shape[axis] = 1;
    else out_shape.erase(out_shape.begin() + axis);
    std::vector<size_m> so = row_major(out_shape);
    so.resize(dims, 0);
    uint32_t cs[8], sa[8], sb[8];
    uint32_t k = orc_collapse_reduce2(shape.data(), so.data(), strides.data(), dims, axis, 0, keep ? 0 : 1, 0xFFFFFFFFu,
                                      cs, sa, sb);
    const uint64_t n = total(out_shape);
    const size_t es = op >= 3 ? 4 : sizeof(T);
    std::vector<uint8_t> out(std::max<uint64_t>(n, 1) * es);
    orc_reduce(op, dtype_code, out.data(), base.data(), strides[axis], shape[axis], k, cs, sa, sb, n, 1);
    out.resize(n * es);
    return out;
}

template <typename T>
static std::vector<uint8_t> oracle_binary(int op, const std::vector<T>& a, const std::vector<size_m>& ash,
                                          const std::vector<T>& b, const std::vector<size_m>& bsh, int dtype_code) {
    std::vector<size_m> ast = row_major(ash), bst = row_major(bsh);
    const int od = (int)std::max(ash.size(), bsh.size());
    uint32_t os[8], ost[8], as_[8], ast2[8], bs_[8], bst2[8];
    orc_broadcast_shapes(ash.data(), ast.data(), (int)ash.size(), bsh.data(), bst.data(), (int)bsh.size(), os, ost, as_,
                         ast2, bs_, bst2);
    uint32_t cs[8], ca[8], cb[8], cr[8];
    uint32_t k = orc_collapse3(as_, ast2, bst2, ost, od, 0x7FFFFFFFu, cs, ca, cb, cr);
    const uint64_t n = total(std::vector<size_m>(os, os + od));
    std::vector<uint8_t> out(std::max<uint64_t>(n, 1) * sizeof(T));
    orc_broadcast(op, dtype_code, out.data(), a.data(), b.data(), k, cr, ca, cb, n, 1);
    out.resize(n * sizeof(T));
    return out;
}

static bool same_bits_f32(const std::vector<uint8_t>& g, const std::vector<uint8_t>& c) {
    if (g.size() != c.size()) return false;
    const float* x = reinterpret_cast<const float*>(g.data());
    const float* y = reinterpret_cast<const float*>(c.data());
    for (size_t i = 0; i < g.size() / 4; ++i) {
        if (std::isnan(x[i]) && std::isnan(y[i])) continue;
        if (std::memcmp(&x[i], &y[i], 4) != 0) return false;
    }
    return true;
}

static std::vector<float> random_ties(size_t n, std::mt19937& rng) {
    std::normal_distribution<float> d(0.f, 1.f);
    std::vector<float> v(n);
    for (auto& x : v) x = std::floor(d(rng) * 8.f) / 8.f;
    return v;
}

static void test_reductions(std::mt19937& rng) {
    std::vector<size_m> shape = {4, 37, 129};
    std::vector<float> host = random_ties(total(shape), rng);
    host[5] = NAN;
    matrix x = matrix::from_host(host.data(), shape, dtype::Float);
    for (int op = 0; op < 5; ++op) {
        for (int axis = 0; axis < 3; ++axis) {
            for (bool keep : {false, true}) {
                matrix y;
                switch (op) {
                    case 0: y = x.sum(axis, keep); break;
                    case 1: y = x.max(axis, keep); break;
                    case 2: y = x.min(axis, keep); break;
                    case 3: y = x.argmax(axis, keep); break;
                    default: y = x.argmin(axis, keep); break;
                }
                y.eval();
                std::vector<uint8_t> g = y.to_host_bytes();
                std::vector<uint8_t> c = oracle_reduce(op, host, shape, x.strides(), axis, keep, 0);
                if (op == 0) {
                    const float* gf = reinterpret_cast<const float*>(g.data());
                    const float* cf = reinterpret_cast<const float*>(c.data());
                    bool ok = g.size() == c.size();
                    for (size_t i = 0; ok && i < c.size() / 4; ++i)
                        ok = (std::isnan(gf[i]) && std::isnan(cf[i])) || std::fabs(gf[i] - cf[i]) <= 1e-3f;
                    EXPECT(ok, "sum axis %d keep %d", axis, keep);
                } else {
                    EXPECT(same_bits_f32(g, c), "reduce op %d axis %d keep %d", op, axis, keep);
                }
                const std::vector<size_m>& s = y.shape();
                EXPECT(s.size() == (keep ? 3u : 2u), "output rank");
            }
        }
    }
    // a transposed view (strided input) and a full reduction
    matrix xt = x.transpose(0, 2);
    matrix yt = xt.argmax(1);
    yt.eval();
    EXPECT(yt.to_host_bytes() == oracle_reduce(3, host, xt.shape(), xt.strides(), 1, false, 0), "argmax of a transpose");
    matrix all = x.max(0).max(0).max(0);
    all.eval();
    std::vector<float> a = all.to_host<float>();
    float ref = -3.4e38f;
    for (float v : host) ref = (ref < v) ? v : ref;
    EXPECT(a.size() == 1 && a[0] == ref, "global max");
    std::vector<int32_t> ih(total(shape));
    for (auto& v : ih) v = (int32_t)(rng() & 0x7FFFFFFF) - (1 << 30);
    matrix xi = matrix::from_host(ih.data(), shape, dtype::Int32);
    matrix si = xi.sum();
    si.eval();
    int32_t want = 0;
    for (auto v : ih) want = (int32_t)((uint32_t)want + (uint32_t)v);
    EXPECT(si.to_host<int32_t>()[0] == want, "int32 full sum wraps like the reference");
}

static void test_binary(std::mt19937& rng) {
    std::vector<size_m> ash = {4, 1, 129}, bsh = {1, 37, 129};
    std::vector<float> a = random_ties(total(ash), rng), b = random_ties(total(bsh), rng);
    for (auto& v : b)
        if (v == 0.f) v = 0.5f;
    matrix A = matrix::from_host(a.data(), ash, dtype::Float);
    matrix B = matrix::from_host(b.data(), bsh, dtype::Float);
    matrix r[6] = {A + B, A - B, A * B, A / B, matrix::max(A, B), matrix::min(A, B)};
    for (int op = 0; op < 6; ++op) {
        r[op].eval();
        EXPECT(r[op].shape() == std::vector<size_m>({4, 37, 129}), "broadcast shape");
        EXPECT(same_bits_f32(r[op].to_host_bytes(), oracle_binary(op, a, ash, b, bsh, 0)), "binary op %d", op);
    }
    std::vector<int32_t> ia(total(ash)), ib(total(bsh));
    for (auto& v : ia) v = (int32_t)rng();
    for (auto& v : ib) v = (int32_t)(rng() | 1);
    matrix IA = matrix::from_host(ia.data(), ash, dtype::Int32), IB = matrix::from_host(ib.data(), bsh, dtype::Int32);
    matrix prod = IA * IB;
    prod.eval();
    EXPECT(prod.to_host_bytes() == oracle_binary(2, ia, ash, ib, bsh, 3), "int32 mul wraps");
    // incompatible shapes throw std::invalid_argument, as Matrix.mm:220 does
    bool threw = false;
    try {
        std::vector<float> c(5 * 7);
        matrix C = matrix::from_host(c.data(), {5, 7}, dtype::Float);
        matrix bad = C + B;
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    EXPECT(threw, "incompatible broadcast throws invalid_argument");
    threw = false;
    try {
        matrix bad = A.sum(3);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    EXPECT(threw, "axis out of range throws invalid_argument");
}

// the softmax trace, unfused (eval) and fused (compile + execute), with the leaf changed between
// executes (the recorded graph is replayed on the new data)
static void test_trace(std::mt19937& rng) {
    const std::vector<size_m> shape = {64, 4096};
    std::vector<float> host(total(shape));
    std::normal_distribution<float> d(0.f, 2.f);
    for (auto& v : host) v = d(rng);
    matrix x = matrix::from_host(host.data(), shape, dtype::Float);
    auto build = [](const matrix& in) {
        matrix m = in.max(-1, true);
        matrix e = matrix::exp(in - m);
        return e / e.sum(-1, true);
    };
    auto reference = [&](const std::vector<float>& h) {
        std::vector<float> y(h.size());
        for (size_t r = 0; r < shape[0]; ++r) {
            const float* row = &h[r * shape[1]];
            float m = -3.4e38f;
            for (size_t c = 0; c < shape[1]; ++c) m = (m < row[c]) ? row[c] : m;
            double s = 0;
            for (size_t c = 0; c < shape[1]; ++c) s += std::exp((double)row[c] - m);
            for (size_t c = 0; c < shape[1]; ++c) y[r * shape[1] + c] = (float)(std::exp((double)row[c] - m) / s);
        }
        return y;
    };
    auto close = [](const std::vector<float>& g, const std::vector<float>& c) {
        if (g.size() != c.size()) return false;
        for (size_t i = 0; i < g.size(); ++i)
            if (!(std::fabs(g[i] - c[i]) <= 1e-5f * std::fabs(c[i]) + 1e-30f)) return false;
        return true;
    };
    matrix unfused = build(x);
    unfused.eval();
    EXPECT(std::string(unfused.tape()->name()) == "Division", "eval() keeps the five primitives");
    EXPECT(close(unfused.to_host<float>(), reference(host)), "unfused softmax trace");

    matrix fused = build(x);
    fused.compile();
    EXPECT(std::string(fused.tape()->name()) == "FusedSoftmax", "compile() fuses the softmax trace");
    fused.execute();
    EXPECT(close(fused.to_host<float>(), reference(host)), "fused softmax, first execute");
    for (auto& v : host) v = d(rng);
    x.upload(host.data());
    fused.execute();  // replays the recorded graph on the new leaf contents
    EXPECT(close(fused.to_host<float>(), reference(host)), "fused softmax, replayed graph");

    // a reduction graph compiled once, executed twice
    std::vector<size_m> bsh = {1, 4096};
    std::vector<float> bias(4096, 0.25f);
    matrix b = matrix::from_host(bias.data(), bsh, dtype::Float);
    matrix z = (x + b).sum(1);
    z.compile();
    z.execute();
    z.execute();
    std::vector<float> zs = z.to_host<float>();
    bool ok = zs.size() == shape[0];
    for (size_t r = 0; ok && r < shape[0]; ++r) {
        double s = 0, abs = 0;
        for (size_t c = 0; c < shape[1]; ++c) {
            const float v = host[r * shape[1] + c] + 0.25f;
            s += v;
            abs += std::fabs(v);
        }
        ok = std::fabs(zs[r] - s) <= 1e-5 * abs;
    }
    EXPECT(ok, "compiled reduction graph");
}

// operator+ with mixed dtypes inserts astype (promote_types), the pointwise family, equal, sqrt's
// promotion, and mean / rms / norm with the dtypes of the reference's composition
static void test_promotion_and_pointwise(std::mt19937& rng) {
    const std::vector<size_m> ash = {4, 1, 129}, bsh = {1, 37, 129};
    std::vector<int32_t> ai(total(ash));
    for (auto& v : ai) v = (int32_t)(rng() % 2001) - 1000;
    std::vector<float> bf = random_ties(total(bsh), rng);
    matrix A = matrix::from_host(ai.data(), ash, dtype::Int32);
    matrix B = matrix::from_host(bf.data(), bsh, dtype::Float);
    matrix S = A + B;  // Int32 + Float -> Float: astype(Float) of A first
    S.eval();
    EXPECT(S.type() == dtype::Float, "Int32 + Float is Float");
    std::vector<float> got = S.to_host<float>();
    bool ok = got.size() == 4u * 37 * 129;
    for (size_t i = 0; ok && i < 4; ++i)
        for (size_t j = 0; ok && j < 37; ++j)
            for (size_t k = 0; ok && k < 129; ++k) {
                volatile float x = (float)ai[i * 129 + k];
                volatile float r = x + bf[j * 129 + k];
                ok = got[(i * 37 + j) * 129 + k] == r;
            }
    EXPECT(ok, "promoted addition");

    // UInt8 * Int8 -> Int16 (both cast), wrapping in Int16
    std::vector<uint8_t> u8(64);
    std::vector<int8_t> i8(64);
    for (int i = 0; i < 64; ++i) {
        u8[i] = (uint8_t)(rng() & 0xFF);
        i8[i] = (int8_t)(rng() & 0xFF);
    }
    matrix P = matrix::from_host(u8.data(), {64}, dtype::UInt8) * matrix::from_host(i8.data(), {64}, dtype::Int8);
    P.eval();
    EXPECT(P.type() == dtype::Int16, "UInt8 * Int8 is Int16");
    std::vector<int16_t> p16 = P.to_host<int16_t>();
    ok = p16.size() == 64;
    for (int i = 0; ok && i < 64; ++i) ok = p16[i] == (int16_t)((int)u8[i] * (int)i8[i]);
    EXPECT(ok, "Int16 product");

    // Int64 - Int32 -> Int64: Int32 converted inside the op's kernel (no AsType node in front)
    std::vector<int64_t> wide64(64);
    std::vector<int32_t> narrow32(64);
    for (int i = 0; i < 64; ++i) {
        wide64[i] = (int64_t)(rng() % 2000001) - 1000000;
        narrow32[i] = (int32_t)(rng() % 2001) - 1000;
    }
    matrix D64 = matrix::from_host(wide64.data(), {64}, dtype::Int64) - matrix::from_host(narrow32.data(), {64}, dtype::Int32);
    D64.eval();
    EXPECT(D64.type() == dtype::Int64, "Int64 - Int32 is Int64");
    std::vector<int64_t> d64 = D64.to_host<int64_t>();
    ok = d64.size() == 64;
    for (int i = 0; ok && i < 64; ++i) ok = d64[i] == wide64[i] - (int64_t)narrow32[i];
    EXPECT(ok, "Int64 difference with the promotion fused");

    // equal, greater, less, where, floor, full, logical_and
    std::vector<float> x = random_ties(8 * 129, rng), y = random_ties(129, rng);
    for (int k = 0; k < 40; ++k) x[k] = y[k];  // some equal pairs in the first row
    matrix X = matrix::from_host(x.data(), {8, 129}, dtype::Float), Y = matrix::from_host(y.data(), {129}, dtype::Float);
    matrix E = matrix::equal(X, Y), G = matrix::greater(X, Y), L = matrix::less(X, Y), F = matrix::floor(X * Y);
    matrix W = matrix::where(G, X, Y);
    matrix Fu = matrix::full({3, 129}, Y, dtype::Int32);
    matrix LA = matrix::logical_and(G, matrix::less(Y, matrix::scalar(0.5f, dtype::Float)));
    for (matrix* m : {&E, &G, &L, &F, &W, &Fu, &LA}) m->eval();
    EXPECT(E.type() == dtype::Float && G.type() == dtype::Bool && W.type() == dtype::Float && Fu.type() == dtype::Int32,
           "pointwise dtypes");
    std::vector<float> e = E.to_host<float>(), f = F.to_host<float>(), w = W.to_host<float>();
    std::vector<uint8_t> g = G.to_host<uint8_t>(), l = L.to_host<uint8_t>(), la = LA.to_host<uint8_t>();
    std::vector<int32_t> fu = Fu.to_host<int32_t>();
    ok = true;
    for (size_t r = 0; r < 8 && ok; ++r)
        for (size_t c = 0; c < 129 && ok; ++c) {
            const float a = x[r * 129 + c], b = y[c];
            volatile float prod = a * b;
            ok = e[r * 129 + c] == (a == b ? 1.f : 0.f) && g[r * 129 + c] == (a > b) && l[r * 129 + c] == (a < b) &&
                 w[r * 129 + c] == (a > b ? a : b) && f[r * 129 + c] == std::floor((float)prod) &&
                 la[r * 129 + c] == ((a > b) && (b < 0.5f));
        }
    for (size_t r = 0; r < 3 && ok; ++r)
        for (size_t c = 0; c < 129 && ok; ++c) ok = fu[r * 129 + c] == (int32_t)y[c];
    EXPECT(ok, "equal / greater / less / where / floor / full / logical_and");

    // sqrt promotes Int32 to Float and Bool to Float16
    std::vector<int32_t> sq = {0, 1, 2, 4, 9, 1000000, 7, 65536};
    matrix R = matrix::sqrt(matrix::from_host(sq.data(), {8}, dtype::Int32));
    R.eval();
    std::vector<float> rs = R.to_host<float>();
    ok = R.type() == dtype::Float && rs.size() == 8;
    for (int i = 0; ok && i < 8; ++i) ok = rs[i] == std::sqrt((float)sq[i]);
    EXPECT(ok, "sqrt(Int32) is a correctly rounded Float sqrt");
    matrix RB = matrix::sqrt(G);
    EXPECT(RB.type() == dtype::Float16, "sqrt(Bool) is Float16");

    // mean / rms / norm
    const std::vector<size_m> shape = {64, 4096};
    std::vector<float> h(total(shape));
    std::normal_distribution<float> d(0.f, 1.f);
    for (auto& v : h) v = d(rng);
    matrix H = matrix::from_host(h.data(), shape, dtype::Float);
    matrix mean = H.mean(1), rms = H.rms(-1), norm = H.norm(1, true), all = H.mean();
    for (matrix* m : {&mean, &rms, &norm, &all}) m->eval();
    EXPECT(std::string(mean.tape()->name()) == "Mean", "mean is one fused node");
    EXPECT(norm.shape() == std::vector<size_m>({64, 1}), "norm keepdims shape");
    std::vector<float> mv = mean.to_host<float>(), rv = rms.to_host<float>(), nv = norm.to_host<float>();
    ok = true;
    double tot = 0, tabs = 0;
    for (size_t r = 0; r < 64 && ok; ++r) {
        double s = 0, a = 0, q = 0;
        for (size_t c = 0; c < 4096; ++c) {
            const double v = h[r * 4096 + c];
            s += v;
            a += std::fabs(v);
            q += (double)((float)(h[r * 4096 + c] * h[r * 4096 + c]));
        }
        tot += s;
        tabs += a;
        ok = std::fabs(mv[r] - s / 4096) <= 1e-5 * a / 4096 + 1e-7 && std::fabs(rv[r] - std::sqrt(q / 4096)) <= 2e-5 * std::sqrt(q / 4096) &&
             std::fabs(nv[r] - std::sqrt(q)) <= 2e-5 * std::sqrt(q);
    }
    EXPECT(ok, "float mean / rms / norm");
    EXPECT(std::fabs(all.to_host<float>()[0] - tot / h.size()) <= 1e-5 * tabs / h.size() + 1e-7, "mean of all elements");
    std::vector<int32_t> hi(4096);
    for (auto& v : hi) v = (int32_t)rng();
    matrix HI = matrix::from_host(hi.data(), {4096}, dtype::Int32);
    matrix mi = HI.mean(0), ni = HI.norm(0);
    mi.eval();
    ni.eval();
    uint32_t s32 = 0, q32 = 0;
    for (auto v : hi) {
        s32 += (uint32_t)v;
        q32 += (uint32_t)v * (uint32_t)v;
    }
    volatile float fs = (float)(int32_t)s32, fq = (float)(int32_t)q32;
    EXPECT(mi.type() == dtype::Float && mi.to_host<float>()[0] == fs / 4096.0f, "int32 mean: wrapped sum / (float)n");
    EXPECT(ni.to_host<float>()[0] == std::sqrt((float)fq) || (std::isnan(ni.to_host<float>()[0]) && fq < 0),
           "int32 norm: sqrt of the wrapped sum of wrapped squares");
}

// Compiled functions (jit_graph_gpu / multi_jit_graph_gpu): every call hands its own input and output
// buffers to the compiled graph, so calls with different buffers -- including more distinct bindings
// than the executor records, and calls inside a larger expression -- each compute their own result.
static void test_jit(std::mt19937& rng) {
    const std::vector<size_m> shape = {32, 2048};
    std::normal_distribution<float> d(0.f, 2.f);
    auto fill = [&](std::vector<float>& v) {
        for (auto& x : v) x = d(rng);
    };
    auto softmax_ref = [&](const std::vector<float>& h) {
        std::vector<float> y(h.size());
        for (size_t r = 0; r < shape[0]; ++r) {
            const float* row = &h[r * shape[1]];
            float m = -3.4e38f;
            for (size_t c = 0; c < shape[1]; ++c) m = (m < row[c]) ? row[c] : m;
            double s = 0;
            for (size_t c = 0; c < shape[1]; ++c) s += std::exp((double)row[c] - m);
            for (size_t c = 0; c < shape[1]; ++c) y[r * shape[1] + c] = (float)(std::exp((double)row[c] - m) / s);
        }
        return y;
    };
    auto close = [](const std::vector<float>& g, const std::vector<float>& c) {
        if (g.size() != c.size()) return false;
        for (size_t i = 0; i < g.size(); ++i)
            if (!(std::fabs(g[i] - c[i]) <= 1e-5f * std::fabs(c[i]) + 1e-30f)) return false;
        return true;
    };
    std::vector<float> h0(total(shape)), h1(total(shape)), h2(total(shape));
    fill(h0);
    fill(h1);
    fill(h2);
    matrix sample = matrix::from_host(h0.data(), shape, dtype::Float);
    auto f = matrix::jit_graph_gpu(
        [](matrix in) {
            matrix m = in.max(-1, true);
            matrix e = matrix::exp(in - m);
            return e / e.sum(-1, true);
        },
        sample);
    matrix x1 = matrix::from_host(h1.data(), shape, dtype::Float);
    matrix x2 = matrix::from_host(h2.data(), shape, dtype::Float);
    matrix y1 = f(x1);
    EXPECT(std::string(y1.tape()->name()) == "CompiledNode", "a call builds a CompiledNode");
    y1.eval();
    matrix y2 = f(x2);
    y2.eval();
    EXPECT(y1.data() != y2.data(), "each call has its own output buffer");
    EXPECT(close(y1.to_host<float>(), softmax_ref(h1)), "jit call 1 reads its own input");
    EXPECT(close(y2.to_host<float>(), softmax_ref(h2)), "jit call 2 reads its own input");
    // more distinct bindings than the executor records (8): the later calls launch directly
    bool all = true;
    std::vector<matrix> keep;
    for (int k = 0; k < 12; ++k) {
        matrix y = f(k % 2 ? x2 : x1);
        y.eval();
        keep.push_back(y);
    }
    for (int k = 0; k < 12; ++k) all = all && close(keep[k].to_host<float>(), softmax_ref(k % 2 ? h2 : h1));
    EXPECT(all, "twelve calls alternating two inputs, each into its own output");
    EXPECT(close(y1.to_host<float>(), softmax_ref(h1)), "an earlier call's output is left alone");
    // a lazy input and a call inside a larger compiled expression, executed twice with new leaf contents
    std::vector<float> bias(shape[1], 0.5f);
    matrix b = matrix::from_host(bias.data(), {1, shape[1]}, dtype::Float);
    matrix z = f(x1 + b) * matrix::scalar(2.0f, dtype::Float);
    z.compile();
    z.execute();
    auto expect_z = [&](const std::vector<float>& h) {
        std::vector<float> hb(h.size());
        for (size_t i = 0; i < h.size(); ++i) hb[i] = h[i] + 0.5f;
        std::vector<float> y = softmax_ref(hb);
        for (auto& v : y) v *= 2.0f;
        return y;
    };
    EXPECT(close(z.to_host<float>(), expect_z(h1)), "jit call inside a compiled expression");
    fill(h1);
    x1.upload(h1.data());
    z.execute();
    EXPECT(close(z.to_host<float>(), expect_z(h1)), "the enclosing expression replayed on new contents");

    // multi-output: Max and ArgMax of one input fuse into one read
    const std::vector<size_m> qs = {16, 300, 96};
    std::vector<float> q0 = random_ties(total(qs), rng), q1 = random_ties(total(qs), rng);
    q1[7] = NAN;
    matrix qsample = matrix::from_host(q0.data(), qs, dtype::Float);
    auto g = matrix::multi_jit_graph_gpu(
        [](std::vector<matrix> in) { return std::vector<matrix>{in[0].max(1), in[0].argmax(1), in[0].min(1)}; },
        {qsample});
    for (const auto* hq : {&q0, &q1}) {
        matrix qx = matrix::from_host(hq->data(), qs, dtype::Float);
        std::vector<matrix> r = g({qx});
        EXPECT(r.size() == 3 && std::string(r[0].tape()->name()) == "MultiInputCompile", "multi-output call");
        r[1].eval();  // evaluating one output runs the compiled graph for all three
        const std::vector<size_m> st = row_major(qs);
        EXPECT(same_bits_f32(r[0].to_host_bytes(), oracle_reduce(1, *hq, qs, st, 1, false, 0)), "jit max");
        EXPECT(r[1].to_host_bytes() == oracle_reduce(3, *hq, qs, st, 1, false, 0), "jit argmax (fused with max)");
        EXPECT(same_bits_f32(r[2].to_host_bytes(), oracle_reduce(2, *hq, qs, st, 1, false, 0)), "jit min");
    }
    // the same fusion for roots compiled together without a jit
    matrix qx = matrix::from_host(q1.data(), qs, dtype::Float);
    matrix mx = qx.max(1), am = qx.argmax(1);
    matrix::compile({&mx, &am});
    EXPECT(std::string(mx.tape()->name()) == "PairMax" && std::string(am.tape()->name()) == "PairArgMax",
           "compile() of max + argmax roots fuses them");
    matrix::execute({&mx, &am});
    EXPECT(same_bits_f32(mx.to_host_bytes(), oracle_reduce(1, q1, qs, row_major(qs), 1, false, 0)), "fused max");
    EXPECT(am.to_host_bytes() == oracle_reduce(3, q1, qs, row_major(qs), 1, false, 0), "fused argmax");

    // the reference's refusals
    bool threw = false;
    try {
        matrix::jit_graph_gpu([](matrix in) { return in; }, sample);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    EXPECT(threw, "a graph whose output is its input is refused (head-tail collision)");
    threw = false;
    try {
        f(matrix::from_host(h1.data(), {shape[1], shape[0]}, dtype::Float));
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    EXPECT(threw, "an input whose layout differs from the sample's is refused");
}

// Ranged and global reductions (flatten(start, end).op(start, keepdims)), flatten's copy of a
// non-contiguous range, the arange generator, arctan2 / arcsin
static void test_ranged_and_generators(std::mt19937& rng) {
    const std::vector<size_m> shape = {6, 7, 33, 5};
    std::vector<float> host = random_ties(total(shape), rng);
    host[11] = NAN;
    matrix x = matrix::from_host(host.data(), shape, dtype::Float);
    // x.sum(1, 2) == x.flatten(1, 2).sum(1): the oracle reduces the same data viewed as [6, 231, 5]
    const std::vector<size_m> fl = {6, 7 * 33, 5};
    matrix s = x.sum(1, 2);
    EXPECT(s.shape() == std::vector<size_m>({6, 5}), "sum(1, 2) shape");
    std::vector<uint8_t> want = oracle_reduce(0, host, fl, row_major(fl), 1, false, 0);
    std::vector<float> g = s.to_host<float>(), w(want.size() / 4);
    std::memcpy(w.data(), want.data(), want.size());
    bool ok = g.size() == w.size();
    for (size_t i = 0; ok && i < g.size(); ++i) ok = (std::isnan(g[i]) && std::isnan(w[i])) || std::fabs(g[i] - w[i]) <= 1e-3f;
    EXPECT(ok, "sum(1, 2)");
    matrix mk = x.max(0, 1, true);
    const std::vector<size_m> f01 = {42, 33, 5};
    EXPECT(mk.shape() == std::vector<size_m>({1, 33, 5}), "max(0, 1, keepdims) shape");
    EXPECT(same_bits_f32(mk.to_host_bytes(), oracle_reduce(1, host, f01, row_major(f01), 0, true, 0)), "max(0, 1, keepdims)");
    matrix mn = x.min(2, 3);
    const std::vector<size_m> f23 = {6, 7, 165};
    EXPECT(same_bits_f32(mn.to_host_bytes(), oracle_reduce(2, host, f23, row_major(f23), 2, false, 0)), "min(2, 3)");
    const std::vector<size_m> all = {(size_m)total(shape)};
    EXPECT(same_bits_f32(x.max().to_host_bytes(), oracle_reduce(1, host, all, {1}, 0, false, 0)), "max()");
    EXPECT(same_bits_f32(x.min().to_host_bytes(), oracle_reduce(2, host, all, {1}, 0, false, 0)), "min()");
    // a transposed view: axes 0..1 of [7, 6, 33, 5] do not chain, so flatten copies first
    matrix xt = x.transpose(0, 1);
    std::vector<float> ht(host.size());
    for (size_t a = 0; a < 6; ++a)
        for (size_t b = 0; b < 7; ++b)
            for (size_t r = 0; r < 33 * 5; ++r) ht[(b * 6 + a) * 165 + r] = host[(a * 7 + b) * 165 + r];
    matrix ft = xt.max(0, 1);
    EXPECT(same_bits_f32(ft.to_host_bytes(), oracle_reduce(1, ht, f01, row_major(f01), 0, false, 0)),
           "max(0, 1) of a transposed view (flatten copies)");
    // integers: the global sum wraps like the reference's T accumulator
    std::vector<int32_t> hi(total(shape));
    std::uniform_int_distribution<int32_t> di(-(1 << 30), 1 << 30);
    for (auto& v : hi) v = di(rng);
    matrix xi = matrix::from_host(hi.data(), shape, dtype::Int32);
    int32_t wsum = 0;
    orc_sum_flat(3, &wsum, hi.data(), hi.size());
    EXPECT(xi.sum().to_host<int32_t>()[0] == wsum, "int32 sum() wraps as the reference's loop");

    // arange: float, half, integers with negative steps; Bool refused; the empty range
    struct Case { double a, b, c; dtype t; int code; };
    const Case cases[] = {{0, 10, 1, dtype::Float, 0}, {-3.5, 1000, 0.1, dtype::Float, 0}, {0, 300, 0.5, dtype::Float16, 1},
                          {5, -100, -3, dtype::Int32, 3}, {3, 250, 1, dtype::UInt8, 2}, {250, 0, -1, dtype::Int16, 4},
                          {0, 1e6, 7, dtype::Int64, 11}, {1, 1, 1, dtype::Float, 0}};
    for (const Case& c : cases) {
        matrix r = matrix::arange(c.a, c.b, c.c, c.t);
        const uint64_t n = r.total_size();
        EXPECT(n == (uint64_t)std::max(0.0, std::ceil((c.b - c.a) / c.c)), "arange length");
        std::vector<uint8_t> got = r.to_host_bytes();
        const size_t es = mtx::dtype_size(c.t);
        std::vector<uint8_t> a(8), st(8), exp(std::max<uint64_t>(n, 1) * es);
        switch (c.t) {
            case dtype::Float: { float u = (float)c.a, v = (float)c.c; std::memcpy(a.data(), &u, 4); std::memcpy(st.data(), &v, 4); break; }
            case dtype::Float16: { _Float16 u = (_Float16)c.a, v = (_Float16)c.c; std::memcpy(a.data(), &u, 2); std::memcpy(st.data(), &v, 2); break; }
            case dtype::Int32: { int32_t u = (int32_t)c.a, v = (int32_t)c.c; std::memcpy(a.data(), &u, 4); std::memcpy(st.data(), &v, 4); break; }
            case dtype::UInt8: { uint8_t u = (uint8_t)c.a, v = (uint8_t)c.c; std::memcpy(a.data(), &u, 1); std::memcpy(st.data(), &v, 1); break; }
            case dtype::Int16: { int16_t u = (int16_t)c.a, v = (int16_t)c.c; std::memcpy(a.data(), &u, 2); std::memcpy(st.data(), &v, 2); break; }
            default: { int64_t u = (int64_t)c.a, v = (int64_t)c.c; std::memcpy(a.data(), &u, 8); std::memcpy(st.data(), &v, 8); break; }
        }
        orc_arange(c.code, exp.data(), a.data(), st.data(), n);
        exp.resize(n * es);
        EXPECT(got == exp, "arange(%g, %g, %g) bit-exact", c.a, c.b, c.c);
    }
    bool threw = false;
    try {
        matrix::arange(0, 4, 1, dtype::Bool);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    EXPECT(threw, "arange refuses Bool");

    // arctan2 (a broadcast operand) and arcsin, against the C library within 3 ulp
    std::vector<float> ya(64 * 33), xb(33);
    std::normal_distribution<float> d(0.f, 3.f);
    for (auto& v : ya) v = d(rng);
    for (auto& v : xb) v = d(rng);
    matrix A = matrix::from_host(ya.data(), {64, 33}, dtype::Float), B = matrix::from_host(xb.data(), {33}, dtype::Float);
    std::vector<float> at = matrix::arctan2(A, B).to_host<float>();
    std::vector<float> as = matrix::arcsin(A * matrix::scalar(0.3f, dtype::Float)).to_host<float>();
    auto ulps = [](float p, float q) {
        int32_t i, j;
        std::memcpy(&i, &p, 4);
        std::memcpy(&j, &q, 4);
        return std::abs((int64_t)i - (int64_t)j);
    };
    bool at_ok = at.size() == ya.size(), as_ok = as.size() == ya.size();
    for (size_t i = 0; at_ok && i < at.size(); ++i) at_ok = ulps(at[i], std::atan2(ya[i], xb[i % 33])) <= 3;
    for (size_t i = 0; as_ok && i < as.size(); ++i) {
        const float w2 = std::asin(ya[i] * 0.3f);
        as_ok = (std::isnan(as[i]) && std::isnan(w2)) || ulps(as[i], w2) <= 3;
    }
    EXPECT(at_ok, "arctan2 with a broadcast operand");
    EXPECT(as_ok, "arcsin");
    EXPECT(matrix::arctan2(xi, xi).type() == dtype::Float, "arctan2 of Int32 inputs casts them to Float");
}

// Runs one test function; an exception counts as a failure with its message instead of ending the run.
template <typename Fn>
static void run_test(const char* name, Fn&& fn) {
    try {
        fn();
    } catch (const std::exception& e) {
        ++checks;
        ++failures;
        std::printf("FAIL %s: exception: %s\n", name, e.what());
    }
}

int main() {
    std::setvbuf(stdout, nullptr, _IOLBF, 0);
    mtx::init(0);
    std::mt19937 rng(1234);
    run_test("reductions", [&] { test_reductions(rng); });
    run_test("binary", [&] { test_binary(rng); });
    run_test("trace", [&] { test_trace(rng); });
    run_test("promotion_and_pointwise", [&] { test_promotion_and_pointwise(rng); });
    run_test("jit", [&] { test_jit(rng); });
    run_test("ranged_and_generators", [&] { test_ranged_and_generators(rng); });
    std::printf("host mirror: %d checks, %d failures\n", checks, failures);
    return failures ? 1 : 0;
}
