// Multi-GPU exchange of the hot path: one NCCL communicator per GPU (one process or host thread per
// GPU), used when a reduction's reduced axis is the one sharded across the GPUs of a node (benchmark
// configs 4 and 5b).  The reference runs on one Metal device (Mods/GPUManager.h:53-54) and has no
// counterpart; this is the multi-GPU half of the device layer that replaces GPUManager.
//
// A sharded reduction runs in three steps, all enqueued on the calling thread's stream:
//   1. every rank reduces its own slice of the axis with the single-GPU kernels (mtxc_reduce, or
//      mtxc_reduce_pair for ArgMax / ArgMin, which also keeps the extreme values), writing straight
//      into its own slot of the communicator's gather buffer;
//   2. one in-place NCCL all-gather (grouped with a second one for the indices) gives every rank every
//      rank's partials, in rank order;
//   3. mtxc_merge_partials merges them in rank order: ordered float sums, first shard wins ties,
//      global first index for ArgMax / ArgMin.
// The all-gather + ordered merge is this library's all-reduce.  It moves nranks x outputs states per
// rank instead of a ring's 2 x outputs, which for the per-shard partials of a reduction (one value per
// output) is a few KB; in exchange every rank computes the identical, deterministic result, and Max /
// ArgMax keep the reference's first-index rule across GPUs, which an NCCL MAX reduction would not.
//
// NCCL is loaded at run time (dlopen), reusing the copy already in the process (PyTorch's) when there
// is one, so the library itself has no link-time NCCL dependency and a one-rank communicator needs no
// NCCL at all.
//
// Peer-memory exchange.  When every rank drives its own GPU of one node, steps 2 and 3 run as ONE kernel
// over NVLink instead of an NCCL all-gather followed by a merge launch: at mtxc_comm_init each rank
// allocates an exchange buffer and maps every other rank's (CUDA IPC handles, passed around once through
// NCCL), and exchange_merge_kernel then (a) stores this rank's partials into its slot of every rank's
// buffer, (b) releases a per-block flag carrying the call's generation in every rank's buffer, (c) waits,
// boundedly, until every rank's flag for that block has arrived in its own buffer, and (d) merges its slice
// of the outputs in rank order from its own buffer.  Each of the fixed kExchBlocks blocks keeps its own
// generation counter in device memory, so consecutive calls (also when replayed from a CUDA graph) use
// alternating slots and no rank can overwrite data a slower rank has not merged yet: a rank starts call
// g + 2 only after call g + 1 saw every rank's data, which every rank sends after finishing call g.  A wait
// that runs out (a rank that never arrives) sets an error flag that mtxc_comm_status reports and returns,
// so no kernel of this library waits forever.  MTXC_COMM_PEER=0 keeps the NCCL path.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "merge.cuh"
#include "mtxc_internal.cuh"

namespace mtxc {
namespace {

struct NcclApi {
    bool ok = false;
    std::string why;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

NcclApi load_nccl() {
    NcclApi api;
    void* h = nullptr;
    const char* env = std::getenv("MTXC_NCCL_LIBRARY");
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy the process already has
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        const char* e = dlerror();
        api.why = std::string("cannot load NCCL (libnccl.so.2): ") + (e ? e : "not found");
        return api;
    }
    bool all = true;
    auto sym = [&](auto& fp, const char* name) {
        fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
        if (!fp) {
            all = false;
            api.why = std::string("NCCL library lacks ") + name;
        }
    };
    sym(api.get_unique_id, "ncclGetUniqueId");
    sym(api.init_rank, "ncclCommInitRank");
    sym(api.destroy, "ncclCommDestroy");
    sym(api.all_gather, "ncclAllGather");
    sym(api.group_start, "ncclGroupStart");
    sym(api.group_end, "ncclGroupEnd");
    sym(api.error_string, "ncclGetErrorString");
    api.ok = all;
    return api;
}

const NcclApi& nccl() {
    static const NcclApi api = load_nccl();
    return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
    const NcclApi& api = nccl();
    return fail(MTXC_ERR_COMM, std::string(what) + ": " + (api.error_string ? api.error_string(r) : "NCCL error") +
                                   " (ncclResult_t " + std::to_string((int)r) + ")");
}

size_t dtype_bytes(int dtype) {
    size_t b = 0;
    dispatch_dtype(dtype, [&](auto* tag) { b = sizeof(*tag); });
    return b;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

constexpr size_t kDefaultCommBytes = size_t(16) << 20;
constexpr int kMaxRanks = 256;  // mtxc_merge_partials' limit on parts

// peer-memory exchange
constexpr int kMaxPeerRanks = 16;    // one node
constexpr int kExchBlocks = 32;      // fixed grid: every call runs the same blocks (per-block generations)
constexpr int kExchThreads = 256;
constexpr uint64_t kDefaultSpinLimit = uint64_t(1) << 22;  // polls of a flag, each followed by a short sleep
constexpr size_t kMinMultiRankBytes = size_t(64) << 10;    // the setup's all-gathers of per-rank cards

// Byte offsets within every rank's exchange buffer (the same layout on all ranks).
struct ExchLayout {
    uint64_t flags = 0;    // uint32 [nranks][kExchBlocks]: the last generation rank r delivered for block b
    uint64_t gens = 0;     // uint32 [kExchBlocks]: this rank's generation per block
    uint64_t err = 0;      // int32: a wait ran out
    uint64_t stage_v = 0;  // this rank's partial values (the local reduction's output)
    uint64_t stage_i = 0;  // and indices
    uint64_t slots_v = 0;  // [2][nranks] value slots of slot_v bytes
    uint64_t slots_i = 0;  // [2][nranks] index slots of slot_i bytes
    uint64_t slot_v = 0, slot_i = 0;
    uint64_t capacity = 0;  // outputs per slot
    uint64_t total = 0;
};

ExchLayout exch_layout(int nranks, size_t budget) {
    ExchLayout L;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = off;
        off += align256(bytes);
        return at;
    };
    L.flags = take((uint64_t)nranks * kExchBlocks * 4);
    L.gens = take(kExchBlocks * 4);
    L.err = take(4);
    const uint64_t fixed = off;
    // values up to 8 bytes and int32 indices, for the staging area and 2 x nranks slots
    L.capacity = budget > fixed ? (budget - fixed) / ((2 * (uint64_t)nranks + 1) * 12 + 512) : 0;
    L.slot_v = align256(L.capacity * 8);
    L.slot_i = align256(L.capacity * 4);
    L.stage_v = take(L.slot_v);
    L.stage_i = take(L.slot_i);
    L.slots_v = off;
    off += 2 * (uint64_t)nranks * L.slot_v;
    L.slots_i = off;
    off += 2 * (uint64_t)nranks * L.slot_i;
    L.total = off;
    return L;
}

}  // namespace

// The calling thread's communicator: ranks, the NCCL handle (none for one rank) and the gather buffer
// (allocated once, in mtxc_comm_init, so the exchange itself never allocates).
struct CommState {
    int nranks = 1;
    int rank = 0;
    int device = -1;
    ncclComm_t comm = nullptr;
    void* buf = nullptr;
    size_t bytes = 0;
    // peer-memory exchange (every rank's exchange buffer, as mapped in this process; peer[rank] is own)
    bool peer = false;
    char* xbuf = nullptr;
    char* peers[kMaxPeerRanks] = {};
    ExchLayout lay;
    uint64_t spin_limit = kDefaultSpinLimit;
};

namespace {
void close_peers(CommState* s) {
    for (int r = 0; r < kMaxPeerRanks; ++r)
        if (s->peers[r] && s->peers[r] != s->xbuf) cudaIpcCloseMemHandle(s->peers[r]);
    for (auto& p : s->peers) p = nullptr;
    if (s->xbuf) cudaFree(s->xbuf);
    s->xbuf = nullptr;
    s->peer = false;
}
}  // namespace

void comm_release() {
    ThreadCtx& c = ctx();
    CommState* s = c.comm;
    if (!s) return;
    c.comm = nullptr;
    cudaSetDevice(s->device);
    cudaStreamSynchronize(c.stream());
    close_peers(s);
    if (s->comm && nccl().destroy) nccl().destroy(s->comm);
    if (s->buf) cudaFree(s->buf);
    delete s;
}

namespace {

// In-place all-gather of `bytes` per rank: rank r's bytes sit at base + r * bytes on entry (its own slot)
// and every rank's slot is filled on exit.
int gather_slots(const CommState& s, void* base, size_t bytes, cudaStream_t st) {
    if (s.nranks == 1 || bytes == 0) return MTXC_OK;
    char* b = static_cast<char*>(base);
    ncclResult_t r = nccl().all_gather(b + (size_t)s.rank * bytes, b, bytes, ncclInt8, s.comm, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return MTXC_OK;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct ExchArgs {
    void* dst;
    int32_t* dst_idx;
    char* peers[kMaxPeerRanks];  // every rank's exchange buffer as mapped here
    ExchLayout lay;
    uint64_t outputs;
    uint64_t spin_limit;
    uint32_t nranks;
    uint32_t rank;
    int64_t offsets[kMaxPeerRanks];
};

// One launch of kExchBlocks blocks: block b owns outputs [b * per, (b + 1) * per) on every rank.
template <int OP, typename T>
__global__ void __launch_bounds__(kExchThreads) exchange_merge_kernel(const ExchArgs a) {
    constexpr bool kArg = OP == MTXC_REDUCE_ARGMAX || OP == MTXC_REDUCE_ARGMIN;
    const uint32_t b = blockIdx.x;
    char* own = a.peers[a.rank];
    uint32_t* gens = reinterpret_cast<uint32_t*>(own + a.lay.gens);
    __shared__ uint32_t s_gen;
    if (threadIdx.x == 0) s_gen = gens[b] + 1u;
    __syncthreads();
    const uint32_t g = s_gen;
    const uint64_t par = g & 1u;
    const uint64_t per = (a.outputs + gridDim.x - 1) / gridDim.x;
    const uint64_t lo = min(a.outputs, (uint64_t)b * per), hi = min(a.outputs, lo + per);
    const T* sv = reinterpret_cast<const T*>(own + a.lay.stage_v);
    const int32_t* si = reinterpret_cast<const int32_t*>(own + a.lay.stage_i);
    const uint64_t my_slot = par * a.nranks + a.rank;
    // (a) this rank's partials into its slot of every rank's buffer, its own included
    for (uint32_t r = 0; r < a.nranks; ++r) {
        T* dv = reinterpret_cast<T*>(a.peers[r] + a.lay.slots_v + my_slot * a.lay.slot_v);
        int32_t* di = reinterpret_cast<int32_t*>(a.peers[r] + a.lay.slots_i + my_slot * a.lay.slot_i);
        for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            dv[i] = sv[i];
            if constexpr (kArg) di[i] = si[i];
        }
    }
    __threadfence_system();
    __syncthreads();
    // (b) this block's part of generation g has arrived at every rank
    if (threadIdx.x < a.nranks) {
        uint32_t* f = reinterpret_cast<uint32_t*>(a.peers[threadIdx.x] + a.lay.flags) + (uint64_t)a.rank * kExchBlocks + b;
        st_release_sys(f, g);
    }
    // (c) wait, boundedly, for every rank's part of generation g here
    if (threadIdx.x < a.nranks) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(own + a.lay.flags) + (uint64_t)threadIdx.x * kExchBlocks + b;
        uint64_t n = 0;
        while ((int32_t)(ld_acquire_sys(f) - g) < 0) {
            if (++n > a.spin_limit) {
                atomicExch(reinterpret_cast<int*>(own + a.lay.err), 1);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    // (d) the ordered merge of this block's outputs from this rank's own slots
    const T* mv = reinterpret_cast<const T*>(own + a.lay.slots_v + par * a.nranks * a.lay.slot_v);
    const int32_t* mi = reinterpret_cast<const int32_t*>(own + a.lay.slots_i + par * a.nranks * a.lay.slot_i);
    for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x)
        merge_one<OP, T>(a.dst, a.dst_idx, mv + i, a.lay.slot_v / sizeof(T), kArg ? mi + i : nullptr, a.lay.slot_i / 4,
                         a.nranks, a.offsets, i);
    if (threadIdx.x == 0) gens[b] = g;
}

template <typename T>
int launch_exchange(int op, const ExchArgs& a, cudaStream_t st) {
    switch (op) {
        case MTXC_REDUCE_SUM: exchange_merge_kernel<MTXC_REDUCE_SUM, T><<<kExchBlocks, kExchThreads, 0, st>>>(a); break;
        case MTXC_REDUCE_MAX: exchange_merge_kernel<MTXC_REDUCE_MAX, T><<<kExchBlocks, kExchThreads, 0, st>>>(a); break;
        case MTXC_REDUCE_MIN: exchange_merge_kernel<MTXC_REDUCE_MIN, T><<<kExchBlocks, kExchThreads, 0, st>>>(a); break;
        case MTXC_REDUCE_ARGMAX: exchange_merge_kernel<MTXC_REDUCE_ARGMAX, T><<<kExchBlocks, kExchThreads, 0, st>>>(a); break;
        default: exchange_merge_kernel<MTXC_REDUCE_ARGMIN, T><<<kExchBlocks, kExchThreads, 0, st>>>(a); break;
    }
    return check_launch("exchange_merge_kernel");
}

// Enqueues the exchange and ordered merge of the partials already in this rank's staging area.
int peer_exchange(CommState& s, int op, int dtype, void* dst, int32_t* dst_idx, uint64_t outputs,
                  const int64_t* index_offsets, cudaStream_t st) {
    ExchArgs a{};
    a.dst = dst;
    a.dst_idx = dst_idx;
    for (int r = 0; r < s.nranks; ++r) a.peers[r] = s.peers[r];
    a.lay = s.lay;
    a.outputs = outputs;
    a.spin_limit = s.spin_limit;
    a.nranks = (uint32_t)s.nranks;
    a.rank = (uint32_t)s.rank;
    for (int r = 0; r < s.nranks && index_offsets; ++r) a.offsets[r] = index_offsets[r];
    int rc = MTXC_OK;
    dispatch_dtype(dtype, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        rc = launch_exchange<T>(op, a, st);
    });
    return rc;
}

// Sets up the peer-memory exchange (every rank must call this, in mtxc_comm_init): allocate and clear this
// rank's exchange buffer, share its IPC handle and the rank's device UUID through NCCL, map every other
// rank's buffer, and agree: the exchange is used only if every rank succeeded and the ranks' devices are
// all distinct (kernels that wait on one another must never share a GPU).
void setup_peer(CommState& s, size_t budget, cudaStream_t st) {
    const char* env = std::getenv("MTXC_COMM_PEER");
    const bool wanted = !(env && env[0] == '0');
    if (const char* sl = std::getenv("MTXC_COMM_SPIN_LIMIT")) {
        const long long v = std::strtoll(sl, nullptr, 10);
        if (v > 0) s.spin_limit = (uint64_t)v;
    }
    struct Card {
        cudaIpcMemHandle_t handle;
        char uuid[16];
        uint64_t total;
        int32_t ok;
        int32_t pad;
    };
    static_assert(sizeof(Card) % 8 == 0, "card size");
    const int n = s.nranks;
    Card mine{};
    s.lay = exch_layout(n, budget);
    bool ok = wanted && n <= kMaxPeerRanks && s.lay.capacity > 0;
    if (ok) ok = cudaMalloc(&s.xbuf, s.lay.total) == cudaSuccess;
    if (ok) ok = cudaMemset(s.xbuf, 0, s.lay.total) == cudaSuccess;
    if (ok) ok = cudaIpcGetMemHandle(&mine.handle, s.xbuf) == cudaSuccess;
    cudaDeviceProp prop{};
    if (ok) ok = cudaGetDeviceProperties(&prop, s.device) == cudaSuccess;
    if (ok) std::memcpy(mine.uuid, &prop.uuid, 16);
    mine.total = s.lay.total;
    mine.ok = ok ? 1 : 0;
    cudaGetLastError();  // a failed step above leaves no sticky error: the NCCL path stays
    // every rank's card, in rank order, through the gather buffer (the same collective on every rank)
    std::vector<Card> cards(n);
    bool shared = (size_t)n * sizeof(Card) <= s.bytes;
    if (shared) {
        char* b = static_cast<char*>(s.buf);
        shared = cudaMemcpy(b + (size_t)s.rank * sizeof(Card), &mine, sizeof(Card), cudaMemcpyHostToDevice) == cudaSuccess;
        // the all-gather runs whatever happened above, so every rank takes the same collective steps
        const bool gathered = gather_slots(s, b, sizeof(Card), st) == MTXC_OK;
        shared = shared && gathered && cudaStreamSynchronize(st) == cudaSuccess &&
                 cudaMemcpy(cards.data(), b, (size_t)n * sizeof(Card), cudaMemcpyDeviceToHost) == cudaSuccess;
    }
    bool all = shared;
    for (int r = 0; r < n && all; ++r) {
        all = cards[r].ok == 1 && cards[r].total == s.lay.total;
        for (int q = 0; q < r && all; ++q) all = std::memcmp(cards[r].uuid, cards[q].uuid, 16) != 0;
    }
    if (all) {
        for (int r = 0; r < n && all; ++r) {
            if (r == s.rank) {
                s.peers[r] = s.xbuf;
                continue;
            }
            void* p = nullptr;
            all = cudaIpcOpenMemHandle(&p, cards[r].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            s.peers[r] = static_cast<char*>(p);
        }
    }
    cudaGetLastError();
    // agree once more: a rank whose mapping failed must make every rank keep the NCCL path
    int32_t mapped = all ? 1 : 0;
    std::vector<int32_t> votes(n, 0);
    bool agreed = false;
    if ((size_t)n * sizeof(int32_t) <= s.bytes) {
        char* b = static_cast<char*>(s.buf);
        bool fine = cudaMemcpy(b + (size_t)s.rank * sizeof(int32_t), &mapped, sizeof(int32_t), cudaMemcpyHostToDevice) ==
                    cudaSuccess;
        const bool gathered = gather_slots(s, b, sizeof(int32_t), st) == MTXC_OK;
        fine = fine && gathered && cudaStreamSynchronize(st) == cudaSuccess &&
               cudaMemcpy(votes.data(), b, (size_t)n * sizeof(int32_t), cudaMemcpyDeviceToHost) == cudaSuccess;
        agreed = fine;
        for (int r = 0; r < n && agreed; ++r) agreed = votes[r] == 1;
    }
    cudaGetLastError();
    if (agreed) s.peer = true;
    else close_peers(&s);
}

int require_comm(CommState*& s, const char* who) {
    if (int rc = require_init()) return rc;
    s = ctx().comm;
    if (!s) return fail(MTXC_ERR_NOT_INITIALIZED, std::string(who) + ": mtxc_comm_init was not called on this thread");
    if (s->device != ctx().device)
        return fail(MTXC_ERR_INVALID_ARGUMENT, std::string(who) + ": the thread's device changed since mtxc_comm_init");
    return MTXC_OK;
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" {

int mtxc_comm_unique_id(void* id, size_t bytes) {
    if (!id || bytes < MTXC_COMM_ID_BYTES)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_comm_unique_id: need a buffer of MTXC_COMM_ID_BYTES bytes");
    static_assert(sizeof(ncclUniqueId) == MTXC_COMM_ID_BYTES, "NCCL unique id size");
    const NcclApi& api = nccl();
    if (!api.ok) return fail(MTXC_ERR_COMM, "mtxc_comm_unique_id: " + api.why);
    ncclUniqueId uid;
    ncclResult_t r = api.get_unique_id(&uid);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id, &uid, sizeof(uid));
    return MTXC_OK;
}

int mtxc_comm_init(int nranks, int rank, const void* id, size_t buffer_bytes) {
    if (int rc = require_init()) return rc;
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_comm_init: need 1 <= nranks <= 256 and 0 <= rank < nranks");
    if (nranks > 1 && !id) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_comm_init: null unique id");
    ThreadCtx& c = ctx();
    if (c.comm) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_comm_init: this thread already has a communicator");
    const NcclApi& api = nccl();
    if (nranks > 1 && !api.ok) return fail(MTXC_ERR_COMM, "mtxc_comm_init: " + api.why);
    auto* s = new CommState();
    s->nranks = nranks;
    s->rank = rank;
    s->device = c.device;
    s->bytes = align256(buffer_bytes ? buffer_bytes : kDefaultCommBytes);
    if (nranks > 1) s->bytes = std::max<size_t>(s->bytes, kMinMultiRankBytes);  // room for the setup exchange
    cudaError_t err = cudaMalloc(&s->buf, s->bytes);
    if (err != cudaSuccess) {
        delete s;
        return cuda_fail(err, "cudaMalloc(communicator buffer)");
    }
    if (nranks > 1) {
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof(uid));
        ncclResult_t r = api.init_rank(&s->comm, nranks, uid, rank);  // blocks until every rank has joined
        if (r != ncclSuccess) {
            cudaFree(s->buf);
            delete s;
            return nccl_fail(r, "ncclCommInitRank");
        }
        setup_peer(*s, buffer_bytes ? buffer_bytes : kDefaultCommBytes, c.stream());
    }
    c.comm = s;
    return MTXC_OK;
}

int mtxc_comm_status(int* peer_exchange, int* timed_out) {
    CommState* s = nullptr;
    if (int rc = require_comm(s, "mtxc_comm_status")) return rc;
    if (peer_exchange) *peer_exchange = s->peer ? 1 : 0;
    if (timed_out) {
        *timed_out = 0;
        if (s->peer) {
            cudaStream_t st = ctx().stream();
            cudaError_t err = cudaStreamSynchronize(st);
            if (err != cudaSuccess) return cuda_fail(err, "cudaStreamSynchronize");
            int32_t flag = 0;
            err = cudaMemcpy(&flag, s->xbuf + s->lay.err, sizeof(flag), cudaMemcpyDeviceToHost);
            if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpy(exchange status)");
            if (flag) {
                *timed_out = 1;
                const int32_t zero = 0;
                err = cudaMemcpy(s->xbuf + s->lay.err, &zero, sizeof(zero), cudaMemcpyHostToDevice);
                if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpy(exchange status)");
            }
        }
    }
    return MTXC_OK;
}

int mtxc_comm_destroy(void) {
    comm_release();
    return MTXC_OK;
}

int mtxc_comm_size(int* nranks, int* rank) {
    if (!nranks || !rank) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_comm_size: null pointer");
    CommState* s = ctx().comm;
    if (!s) return fail(MTXC_ERR_NOT_INITIALIZED, "mtxc_comm_size: mtxc_comm_init was not called on this thread");
    *nranks = s->nranks;
    *rank = s->rank;
    return MTXC_OK;
}

int mtxc_reduce_sharded(int op, int dtype, void* dst, const void* src, uint32_t reduce_stride, uint32_t reduce_len,
                        uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides,
                        const uint32_t* src_strides, const int64_t* index_offsets) {
    CommState* s = nullptr;
    if (int rc = require_comm(s, "mtxc_reduce_sharded")) return rc;
    if (op < MTXC_REDUCE_SUM || op > MTXC_REDUCE_ARGMIN)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_sharded: unknown op");
    const size_t esize = dtype_bytes(dtype);
    if (!esize)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_reduce_sharded: no kernel for dtype ") + dtype_name(dtype));
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_sharded: cdims > MTXC_MAX_DIMS");
    if (cdims && !shape) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_sharded: null metadata pointer");
    const uint64_t outputs = cdims ? product(shape, cdims) : 1;
    if (outputs == 0) return MTXC_OK;
    if (!dst) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_sharded: null buffer");
    const bool arg = op == MTXC_REDUCE_ARGMAX || op == MTXC_REDUCE_ARGMIN;
    if (arg && !index_offsets)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_reduce_sharded: ArgMax / ArgMin need index_offsets (one per rank)");
    const size_t val_slot = (size_t)outputs * esize;
    const size_t idx_slot = arg ? (size_t)outputs * sizeof(int32_t) : 0;
    const size_t val_bytes = align256(val_slot * (size_t)s->nranks);
    // one kernel over peer memory: the local reduction goes to this rank's staging area, then the
    // exchange + ordered merge
    if (s->peer && outputs <= s->lay.capacity) {
        void* sv = s->xbuf + s->lay.stage_v;
        int32_t* si = reinterpret_cast<int32_t*>(s->xbuf + s->lay.stage_i);
        int rc = arg ? mtxc_reduce_pair(op, dtype, sv, si, src, reduce_stride, reduce_len, cdims, shape, dst_strides,
                                        src_strides)
                     : mtxc_reduce(op, dtype, sv, src, reduce_stride, reduce_len, cdims, shape, dst_strides, src_strides);
        if (rc) return rc;
        return peer_exchange(*s, op, dtype, arg ? nullptr : dst, arg ? static_cast<int32_t*>(dst) : nullptr, outputs,
                             index_offsets, ctx().stream());
    }
    const size_t need = val_bytes + idx_slot * (size_t)s->nranks;
    if (need > s->bytes)
        return fail(MTXC_ERR_WORKSPACE, "mtxc_reduce_sharded: the gathered partials need " + std::to_string(need) +
                                            " bytes, more than the communicator's " + std::to_string(s->bytes) +
                                            " (mtxc_comm_init's buffer_bytes)");
    char* vals = static_cast<char*>(s->buf);
    int32_t* idx = arg ? reinterpret_cast<int32_t*>(vals + val_bytes) : nullptr;
    char* my_vals = vals + (size_t)s->rank * val_slot;
    int32_t* my_idx = arg ? idx + (size_t)s->rank * outputs : nullptr;

    // 1. this rank's slice, into its own slots
    int rc = arg ? mtxc_reduce_pair(op, dtype, my_vals, my_idx, src, reduce_stride, reduce_len, cdims, shape, dst_strides,
                                    src_strides)
                 : mtxc_reduce(op, dtype, my_vals, src, reduce_stride, reduce_len, cdims, shape, dst_strides, src_strides);
    if (rc) return rc;
    // 2. every rank's partials, in rank order
    cudaStream_t st = ctx().stream();
    if (s->nranks > 1) {
        ncclResult_t r = nccl().group_start();
        if (r != ncclSuccess) return nccl_fail(r, "ncclGroupStart");
        int grc = gather_slots(*s, vals, val_slot, st);
        if (!grc && arg) grc = gather_slots(*s, idx, idx_slot, st);
        r = nccl().group_end();
        if (grc) return grc;
        if (r != ncclSuccess) return nccl_fail(r, "ncclGroupEnd");
    }
    // 3. ordered merge, identical on every rank
    if (arg) return mtxc_merge_partials(op, dtype, nullptr, static_cast<int32_t*>(dst), vals, idx, index_offsets,
                                        (uint32_t)s->nranks, outputs);
    return mtxc_merge_partials(op, dtype, dst, nullptr, vals, nullptr, nullptr, (uint32_t)s->nranks, outputs);
}

int mtxc_allreduce(int op, int dtype, void* buf, uint64_t count) {
    CommState* s = nullptr;
    if (int rc = require_comm(s, "mtxc_allreduce")) return rc;
    if (op != MTXC_REDUCE_SUM && op != MTXC_REDUCE_MAX && op != MTXC_REDUCE_MIN)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_allreduce: op must be SUM, MAX or MIN");
    const size_t esize = dtype_bytes(dtype);
    if (!esize)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_allreduce: no kernel for dtype ") + dtype_name(dtype));
    if (count == 0) return MTXC_OK;
    if (!buf) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_allreduce: null buffer");
    const size_t slot = (size_t)count * esize;
    if (slot * (size_t)s->nranks > s->bytes)
        return fail(MTXC_ERR_WORKSPACE, "mtxc_allreduce: " + std::to_string(slot * (size_t)s->nranks) +
                                            " bytes to gather, more than the communicator's " + std::to_string(s->bytes));
    if (s->nranks == 1) return MTXC_OK;
    cudaStream_t st = ctx().stream();
    if (s->peer && count <= s->lay.capacity) {
        cudaError_t err = cudaMemcpyAsync(s->xbuf + s->lay.stage_v, buf, slot, cudaMemcpyDeviceToDevice, st);
        if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(D2D)");
        return peer_exchange(*s, op, dtype, buf, nullptr, count, nullptr, st);
    }
    char* vals = static_cast<char*>(s->buf);
    cudaError_t err = cudaMemcpyAsync(vals + (size_t)s->rank * slot, buf, slot, cudaMemcpyDeviceToDevice, st);
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(D2D)");
    if (int rc = gather_slots(*s, vals, slot, st)) return rc;
    return mtxc_merge_partials(op, dtype, buf, nullptr, vals, nullptr, nullptr, (uint32_t)s->nranks, count);
}

}  // extern "C"
