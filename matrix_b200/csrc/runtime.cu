// Runtime: per-thread device / stream / workspace context, memory, copies, errors and CUDA
// graph capture.  Replaces the reference's GPUManager device, queue and thread-local command
// buffer (Mods/GPUManager.h:47-600) and its buffer wrapping (matrix.h:677-680).
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "mtxc_internal.cuh"

namespace mtxc {

ThreadCtx& ctx() {
    thread_local ThreadCtx c;
    return c;
}

int fail(int code, const std::string& msg) {
    ctx().last_error = msg;
    return code;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(MTXC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")");
}

int require_init() {
    ThreadCtx& c = ctx();
    if (c.device < 0) return fail(MTXC_ERR_NOT_INITIALIZED, "mtxc_init was not called on this thread");
    // Other code in the process (another library, another runtime) may have made a different
    // device current on this thread since mtxc_init; launches and copies must go to the bound one.
    int current = -1;
    if (cudaGetDevice(&current) != cudaSuccess || current != c.device) {
        cudaError_t err = cudaSetDevice(c.device);
        if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
    }
    return MTXC_OK;
}

int check_launch(const char* what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, what);
    return MTXC_OK;
}

const char* dtype_name(int dtype) {
    static const char* names[] = {"Float",  "Float16", "UInt8",     "Int32",    "Int16", "UInt32", "UInt16",
                                  "Bool",   "Int8",    "Complex64", "BFloat16", "Int64", "UInt64"};
    if (dtype < 0 || dtype > 12) return "<invalid>";
    return names[dtype];
}

static size_t default_workspace_bytes() {
    size_t mb = 64;
    if (const char* env = std::getenv("MTXC_WORKSPACE_MB")) {
        long v = std::strtol(env, nullptr, 10);
        if (v >= 0) mb = (size_t)v;
    }
    return mb << 20;
}

}  // namespace mtxc

using namespace mtxc;

extern "C" {

int mtxc_abi_version(void) { return MTXC_ABI_VERSION; }

int mtxc_device_count(int* count) {
    if (!count) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_device_count: null pointer");
    cudaError_t err = cudaGetDeviceCount(count);
    if (err != cudaSuccess) {
        *count = 0;
        return cuda_fail(err, "cudaGetDeviceCount");
    }
    return MTXC_OK;
}

int mtxc_init(int device) {
    ThreadCtx& c = ctx();
    if (c.device == device && c.own_stream) return MTXC_OK;
    if (c.device >= 0) mtxc_shutdown();
    cudaError_t err = cudaSetDevice(device);
    if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
    err = cudaStreamCreateWithFlags(&c.own_stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamCreateWithFlags");
    int sms = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(MultiProcessorCount)");
    c.sm_count = sms;
    c.device = device;
    const size_t ws = default_workspace_bytes();
    if (ws) {
        err = cudaMalloc(&c.workspace, ws);
        if (err != cudaSuccess) {
            c.workspace = nullptr;
            return cuda_fail(err, "cudaMalloc(workspace)");
        }
        c.workspace_bytes = ws;
        c.own_workspace = true;
    }
    c.last_error.clear();
    return MTXC_OK;
}

int mtxc_shutdown(void) {
    ThreadCtx& c = ctx();
    if (c.device < 0) return MTXC_OK;
    cudaSetDevice(c.device);
    comm_release();
    noalloc_forget(c.device);
    if (c.own_stream) {
        cudaStreamSynchronize(c.own_stream);
        cudaStreamDestroy(c.own_stream);
    }
    if (c.own_workspace && c.workspace) cudaFree(c.workspace);
    c = ThreadCtx();
    return MTXC_OK;
}

const char* mtxc_last_error(void) { return ctx().last_error.c_str(); }

int mtxc_set_stream(void* stream) {
    if (int rc = require_init()) return rc;
    ctx().user_stream = static_cast<cudaStream_t>(stream);
    ctx().has_user_stream = true;
    return MTXC_OK;
}

int mtxc_use_own_stream(void) {
    if (int rc = require_init()) return rc;
    ctx().user_stream = nullptr;
    ctx().has_user_stream = false;
    return MTXC_OK;
}

void* mtxc_get_stream(void) { return ctx().stream(); }

int mtxc_sync(void) {
    if (int rc = require_init()) return rc;
    cudaError_t err = cudaStreamSynchronize(ctx().stream());
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamSynchronize");
    return MTXC_OK;
}

int mtxc_set_workspace(void* ptr, size_t bytes) {
    if (int rc = require_init()) return rc;
    if ((bytes && !ptr) || (reinterpret_cast<uintptr_t>(ptr) & 255u) || (bytes & 255u))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_set_workspace: pointer and size must be multiples of 256");
    ThreadCtx& c = ctx();
    if (c.own_workspace && c.workspace) {
        cudaError_t err = cudaStreamSynchronize(c.stream());
        if (err != cudaSuccess) return cuda_fail(err, "cudaStreamSynchronize");
        cudaFree(c.workspace);
    }
    c.workspace = ptr;
    c.workspace_bytes = bytes;
    c.own_workspace = false;
    return MTXC_OK;
}

int mtxc_workspace_size(size_t* bytes) {
    if (!bytes) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_workspace_size: null pointer");
    *bytes = ctx().workspace_bytes;
    return MTXC_OK;
}

int mtxc_alloc(size_t bytes, void** dptr) {
    if (int rc = require_init()) return rc;
    if (!dptr) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_alloc: null pointer");
    cudaError_t err = cudaMalloc(dptr, bytes ? bytes : 1);
    if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc");
    return MTXC_OK;
}

int mtxc_free(void* dptr) {
    if (!dptr) return MTXC_OK;
    cudaError_t err = cudaFree(dptr);
    if (err != cudaSuccess) return cuda_fail(err, "cudaFree");
    return MTXC_OK;
}

int mtxc_host_alloc(size_t bytes, void** hptr) {
    if (!hptr) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_host_alloc: null pointer");
    cudaError_t err = cudaMallocHost(hptr, bytes ? bytes : 1);
    if (err != cudaSuccess) return cuda_fail(err, "cudaMallocHost");
    return MTXC_OK;
}

int mtxc_host_free(void* hptr) {
    if (!hptr) return MTXC_OK;
    cudaError_t err = cudaFreeHost(hptr);
    if (err != cudaSuccess) return cuda_fail(err, "cudaFreeHost");
    return MTXC_OK;
}

int mtxc_upload(void* dst, const void* src, size_t bytes) {
    if (int rc = require_init()) return rc;
    if (!bytes) return MTXC_OK;
    if (!dst || !src) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_upload: null pointer");
    cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx().stream());
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(H2D)");
    return MTXC_OK;
}

int mtxc_download(void* dst, const void* src, size_t bytes) {
    if (int rc = require_init()) return rc;
    if (!bytes) return MTXC_OK;
    if (!dst || !src) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_download: null pointer");
    cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx().stream());
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(D2H)");
    return MTXC_OK;
}

int mtxc_copy_device(void* dst, const void* src, size_t bytes) {
    if (int rc = require_init()) return rc;
    if (!bytes) return MTXC_OK;
    if (!dst || !src) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_copy_device: null pointer");
    cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx().stream());
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(D2D)");
    return MTXC_OK;
}

int mtxc_memset(void* dptr, int value, size_t bytes) {
    if (int rc = require_init()) return rc;
    if (!bytes) return MTXC_OK;
    if (!dptr) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_memset: null pointer");
    cudaError_t err = cudaMemsetAsync(dptr, value, bytes, ctx().stream());
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync");
    return MTXC_OK;
}

// ------------------------------------------------------------------------------------------
// Graph capture: compile once, execute many.
// ------------------------------------------------------------------------------------------
int mtxc_graph_begin(void) {
    if (int rc = require_init()) return rc;
    cudaError_t err = cudaStreamBeginCapture(ctx().stream(), cudaStreamCaptureModeThreadLocal);
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamBeginCapture");
    return MTXC_OK;
}

int mtxc_graph_end(void** graph) {
    if (int rc = require_init()) return rc;
    if (!graph) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_graph_end: null pointer");
    cudaGraph_t g = nullptr;
    cudaError_t err = cudaStreamEndCapture(ctx().stream(), &g);
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    err = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphInstantiate");
    *graph = exec;
    return MTXC_OK;
}

int mtxc_graph_launch(void* graph) {
    if (int rc = require_init()) return rc;
    if (!graph) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_graph_launch: null graph");
    cudaError_t err = cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph), ctx().stream());
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphLaunch");
    return MTXC_OK;
}

int mtxc_graph_destroy(void* graph) {
    if (!graph) return MTXC_OK;
    cudaError_t err = cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph));
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphExecDestroy");
    return MTXC_OK;
}

}  // extern "C"
