// The C++ host mirror's multi-GPU calls (mtx::Communicator, mtx::reduce_sharded) on several GPUs, one
// process per GPU: every rank holds a contiguous slice of axis 0 of the same tensor and reduces over that
// axis; every rank's result must equal the CPU oracle's reduction of the whole tensor (the reference's
// CPU eval restated: Matrix.mm:15187-15207 sum, 14894-14914 max, 15038-15058 min, 16279-16302 argmax,
// 16434-16457 argmin).  Bit-exact except float sums, which are within 1e-5 * sum|x| (tests/helpers.py's
// rule).  The tensors put equal extremes on both sides of a shard boundary (the earlier global row must
// win), a column whose only minimum is a later rank's first row, and int32 sums that wrap.  A compiled
// pass (x * x then the sharded sum) is executed, its leaf overwritten and executed again: the recorded
// pass, exchange included, replays with the new contents.
//
// Usage: test_mirror_sharded <rank> <nranks> <id file>.  Rank 0 writes the communicator id to the file;
// the other ranks wait for it (60 s at most).  Prints "<checks> checks, <failures> failures".
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "mtx.hpp"
#include "mtxc.h"

extern "C" {
uint32_t orc_collapse_reduce2(const uint32_t*, const uint32_t*, const uint32_t*, uint32_t, int, int, int, uint64_t,
                              uint32_t*, uint32_t*, uint32_t*);
int orc_reduce(int, int, void*, const void*, uint32_t, uint32_t, uint32_t, const uint32_t*, const uint32_t*,
               const uint32_t*, uint64_t, int);
}

using mtx::dtype;
using mtx::matrix;
using mtx::ReduceOp;
using mtx::size_m;

static int checks = 0, failures = 0;

#define EXPECT(cond, ...)                                      \
    do {                                                       \
        ++checks;                                              \
        if (!(cond)) {                                         \
            ++failures;                                        \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__);   \
            std::printf(__VA_ARGS__);                          \
            std::printf("\n");                                 \
        }                                                      \
    } while (0)

static const std::vector<size_m> kShape = {9, 33, 20};  // axis 0 is sharded
static constexpr size_m kInner = 33 * 20;

// rank r's rows [lo, hi) of n: the first n % world ranks take one row more
static void shard(size_m n, int world, int r, size_m& lo, size_m& hi) {
    const size_m base = n / world, extra = n % world;
    lo = r * base + std::min<size_m>(r, extra);
    hi = lo + base + (r < (int)extra ? 1 : 0);
}

// the oracle's x.op(0) over the whole [9, 33, 20] tensor
template <typename T>
static std::vector<uint8_t> oracle_axis0(int op, const std::vector<T>& x, int code) {
    const uint32_t dims = 3;
    std::vector<size_m> strides = {kInner, 20, 1};
    std::vector<size_m> so = {20, 1, 0};  // the output's row-major strides, padded to the input's dims
    uint32_t cs[8], sa[8], sb[8];
    const uint32_t k = orc_collapse_reduce2(kShape.data(), so.data(), strides.data(), dims, 0, 0, 1, 0xFFFFFFFFu, cs, sa, sb);
    const size_t es = op >= 3 ? 4 : sizeof(T);
    std::vector<uint8_t> out(kInner * es);
    orc_reduce(op, code, out.data(), x.data(), strides[0], kShape[0], k, cs, sa, sb, kInner, 1);
    return out;
}

// float sums: within 1e-5 * sum|x| of the oracle; everything else bit for bit
static void compare(const char* what, int op, const std::vector<uint8_t>& got, const std::vector<uint8_t>& want,
                    const std::vector<float>* xf) {
    EXPECT(got.size() == want.size(), "%s: %zu bytes, want %zu", what, got.size(), want.size());
    if (got.size() != want.size()) return;
    if (op == 0 && xf) {
        const float* g = reinterpret_cast<const float*>(got.data());
        const float* w = reinterpret_cast<const float*>(want.data());
        int bad = 0;
        for (size_m c = 0; c < kInner; ++c) {
            double abs_sum = 0;
            for (size_m r = 0; r < kShape[0]; ++r) abs_sum += std::fabs((double)(*xf)[r * kInner + c]);
            if (!(std::fabs((double)g[c] - (double)w[c]) <= 1e-5 * abs_sum)) ++bad;
        }
        EXPECT(bad == 0, "%s: %d of %u sums outside 1e-5 * sum|x|", what, bad, kInner);
        return;
    }
    EXPECT(std::memcmp(got.data(), want.data(), got.size()) == 0, "%s: not bit-exact", what);
}

static std::string read_id(const std::string& path, int rank, int nranks) {
    if (rank == 0) {
        const std::string id = nranks > 1 ? mtx::Communicator::unique_id() : std::string();
        const std::string tmp = path + ".tmp";
        std::ofstream(tmp, std::ios::binary).write(id.data(), (std::streamsize)id.size());
        std::rename(tmp.c_str(), path.c_str());
        return id;
    }
    for (int i = 0; i < 600; ++i) {
        std::ifstream f(path, std::ios::binary);
        if (f) {
            std::string id((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
            if (id.size() == MTXC_COMM_ID_BYTES) return id;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
    }
    throw std::runtime_error("no communicator id from rank 0");
}

int main(int argc, char** argv) {
    if (argc != 4) {
        std::printf("usage: %s <rank> <nranks> <id file>\n", argv[0]);
        return 2;
    }
    const int rank = std::atoi(argv[1]), nranks = std::atoi(argv[2]);
    mtx::init(rank);
    const std::string id = read_id(argv[3], rank, nranks);
    mtx::Communicator comm(nranks, rank, id);
    std::printf("rank %d peer=%d\n", rank, comm.peer_exchange() ? 1 : 0);

    const size_m n = kShape[0];
    size_m lo, hi;
    shard(n, nranks, rank, lo, hi);
    std::vector<int64_t> first_rows(nranks);
    for (int r = 0; r < nranks; ++r) {
        size_m a, b;
        shard(n, nranks, r, a, b);
        first_rows[r] = a;
    }
    size_m b1, e1;  // the second rank's first row: the boundary the ties straddle
    shard(n, nranks, nranks > 1 ? 1 : 0, b1, e1);
    const size_m b = nranks > 1 ? b1 : 4;

    std::mt19937 gen(11);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::uniform_int_distribution<int32_t> ud(-(1 << 30), 1 << 30);
    std::vector<float> xf(n * kInner);
    std::vector<int32_t> xi(n * kInner);
    for (auto& v : xf) v = std::floor(nd(gen) * 4.f) / 4.f;  // quarter steps: ties
    for (auto& v : xi) v = ud(gen);
    for (size_m c = 0; c < 20; ++c) {
        xf[(b - 1) * kInner + c] = xf[b * kInner + c] = 100.f;    // equal maxima either side of the boundary
        xf[b * kInner + 20 + c] = -100.f;                         // the only minimum: a later rank's first row
        xi[(b - 1) * kInner + 40 + c] = xi[b * kInner + 40 + c] = 0x7fffffff;
        for (size_m r = 0; r < n; ++r) xi[r * kInner + 60 + c] = (1 << 30) + 7;  // 9 (2^30 + 7) wraps
    }
    const matrix lf = matrix::from_host(xf.data() + (size_t)lo * kInner, {hi - lo, 33, 20}, dtype::Float);
    const matrix li = matrix::from_host(xi.data() + (size_t)lo * kInner, {hi - lo, 33, 20}, dtype::Int32);
    const char* names[] = {"sum", "max", "min", "argmax", "argmin"};
    for (int op = 0; op < 5; ++op) {
        char what[96];
        std::snprintf(what, sizeof what, "rank %d float %s(0)", rank, names[op]);
        compare(what, op, mtx::reduce_sharded((ReduceOp)op, lf, first_rows).to_host_bytes(),
                oracle_axis0(op, xf, 0), &xf);
        std::snprintf(what, sizeof what, "rank %d int32 %s(0)", rank, names[op]);
        compare(what, op, mtx::reduce_sharded((ReduceOp)op, li, first_rows).to_host_bytes(),
                oracle_axis0(op, xi, 3), nullptr);
    }
    {  // keepdims: the same values in a [1, 33, 20] result
        const matrix k = mtx::reduce_sharded(ReduceOp::ArgMax, lf, first_rows, true);
        EXPECT(k.shape() == std::vector<size_m>({1, 33, 20}), "rank %d keepdims shape", rank);
        compare("keepdims argmax", 3, k.to_host_bytes(), oracle_axis0(3, xf, 0), nullptr);
    }
    {  // a compiled pass: x * x, then the sharded sum; executed, the leaf overwritten, executed again
        matrix leaf = matrix::from_host(xf.data() + (size_t)lo * kInner, {hi - lo, 33, 20}, dtype::Float);
        matrix y = mtx::reduce_sharded(ReduceOp::Sum, leaf * leaf);
        y.compile();
        for (int pass = 0; pass < 3; ++pass) {
            std::vector<float> x2(xf);
            for (auto& v : x2) v = v * (1.0f + 0.25f * (float)pass);
            leaf.upload(x2.data() + (size_t)lo * kInner);
            std::vector<float> sq(x2.size());
            for (size_t i = 0; i < sq.size(); ++i) sq[i] = x2[i] * x2[i];
            y.execute();  // the first records the pass (exchange included); the others replay it
            char what[64];
            std::snprintf(what, sizeof what, "rank %d compiled sum(x*x) pass %d", rank, pass);
            compare(what, 0, y.to_host_bytes(), oracle_axis0(0, sq, 0), &sq);
        }
    }
    EXPECT(!comm.timed_out(), "rank %d: an exchange gave up waiting", rank);
    comm.barrier();
    std::printf("rank %d: %d checks, %d failures\n", rank, checks, failures);
    return failures ? 1 : 0;
}
