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
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <mutex>

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
};

void comm_release() {
    ThreadCtx& c = ctx();
    CommState* s = c.comm;
    if (!s) return;
    c.comm = nullptr;
    cudaSetDevice(s->device);
    cudaStreamSynchronize(c.stream());
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
    }
    c.comm = s;
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
    char* vals = static_cast<char*>(s->buf);
    cudaStream_t st = ctx().stream();
    cudaError_t err = cudaMemcpyAsync(vals + (size_t)s->rank * slot, buf, slot, cudaMemcpyDeviceToDevice, st);
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(D2D)");
    if (int rc = gather_slots(*s, vals, slot, st)) return rc;
    return mtxc_merge_partials(op, dtype, buf, nullptr, vals, nullptr, nullptr, (uint32_t)s->nranks, count);
}

}  // extern "C"
