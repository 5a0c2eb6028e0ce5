// mtx.hpp -- C++ host mirror of AlanAditya/matrix's API for the reduce / broadcast hot path, on the
// B200 backend (include/mtxc.h).
//
// The reference is a lazy graph library: an op builds a Primitive node and caches the shape metadata
// its backend needs (matrix.h:496-1787, primitives.cpp:57-118); eval() / compile() / execute() walk
// the graph.  This header keeps those names and their meaning for the ops on the hot path:
//   frontends   operator+ - * / with promotion (astype in front), matrix::max / min(a, b), matrix::equal
//               (Matrix.mm:8312-8382, 13363-13376, 14668-14682, 14451-14466)
//               x.sum / max / min / argmax / argmin(axis, keepdims), x.sum()   (Matrix.mm:14784-16335, 15210-15218)
//               x.mean / rms / norm(axis, keepdims) and over all elements    (Matrix.mm:15220-15276)
//               matrix::exp / sqrt(x) with promotion to Float16 or wider      (Matrix.mm:6798-6811, 6934-6947)
//               x.astype(t, make_contig)                                       (Matrix.mm:8384-8398)
//               matrix::greater / less / logical_and / where / floor / full    (Matrix.mm:13572-13593)
//               matrix::arctan2 / arcsin / arange                              (Matrix.mm:13573-13604)
//               x.sum / max / min(start, end, keepdims), x.max(), x.min(), x.flatten(start, end)
//               matrix::scalar(v, t)                                           (a 0-d matrix holding dtype_cast<t>(v))
//   primitives  allocate-or-adopt the output, return before computing under COMPILE_TRACE, run once
//               per pass (`evaluated`), then call the backend (primitives.cpp:2836-2902)
//   evaluation  eval() = compile + execute in one pass; compile() allocates every output and fuses
//               the softmax trace (and Max + ArgMax roots compiled together); execute() runs kernels
//               only -- recorded into a CUDA graph per binding of device pointers, replayed while the
//               binding holds (Matrix.mm:8415-8475); jit_graph_gpu / multi_jit_graph_gpu hand each call's
//               buffers to a compiled graph (Matrix.mm:1076-1149)
//   several GPUs Communicator (mtxc_comm_*) and reduce_sharded: a reduction over an axis sharded across
//               the GPUs of a node, one lazy node per rank (no counterpart in the reference)
// mean / rms / norm build one fused node (mtxc_reduce_stat: one read of x) whose result and dtype are
// those of the reference's composition (sum, scalar division, sqrt); the other frontends build the
// reference's own nodes.
// Errors keep the reference's exception types: std::invalid_argument for shapes and axes
// (Matrix.mm:220), std::runtime_error for everything else (Mods/GPUManager.h:62-71).
//
// Tensors live in device memory (HBM); from_host / to_host move data explicitly, where the
// reference's unified memory needs no copies.  There is no CPU evaluation path: this is the GPU
// backend, and it fails loudly rather than falling back.
#pragma once

#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace mtx {

using size_m = uint32_t;  // Mods/Utils.h:125

// matrix.h:35-51 (the codes are the ABI)
enum class dtype : uint8_t {
    Float = 0, Float16 = 1, UInt8 = 2, Int32 = 3, Int16 = 4, UInt32 = 5, UInt16 = 6, Bool = 7, Int8 = 8,
    Complex64 = 9, BFloat16 = 10, Int64 = 11, UInt64 = 12
};
size_t dtype_size(dtype t);
dtype promote_types(dtype a, dtype b);

// Mods/Utils.h:92-97
enum class EvalType { EVAL_AUTO = 0, EVAL_INSTANTLY = 1, COMPILE_TRACE = 2, EXEC_TRACE = 3 };

// Binds the calling thread to a device (mtxc_init); call once per thread before building graphs.
void init(int device = 0);

// Device memory owned by one or more matrices (the reference's buffer + refCount).  An alias refers to
// memory another Buffer owns (a caller's input handed to a compiled graph) and keeps that owner alive.
struct Buffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    explicit Buffer(size_t n);
    Buffer(void* alias, size_t n, std::shared_ptr<Buffer> owner);
    ~Buffer();
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;

private:
    std::shared_ptr<Buffer> owner_;  // set for an alias, which frees nothing
};

class matrix;

class Primitive {
public:
    virtual ~Primitive() = default;
    bool evaluated = false;
    std::shared_ptr<Buffer> out_buffer;  // the tape's cached output (allocate once, adopt after)
    // DFS: inputs first, then allocate-or-adopt `out`, return under COMPILE_TRACE, run once per pass
    virtual void eval(matrix& out, EvalType eval_type) = 0;
    virtual void clear_trace_checks() = 0;
    virtual std::vector<matrix*> inputs() = 0;
    virtual const char* name() const = 0;
    // device pointers this node writes besides out_buffer (a fused node's sibling outputs): part of the
    // binding a recorded pass is keyed on
    virtual void extra_bindings(std::vector<const void*>&) const {}
};

// Recorded execute passes of one graph, keyed by every device pointer the pass binds (defined in mtx.cpp).
struct GraphCache;

class matrix {
public:
    matrix() = default;
    // leaves
    static matrix from_host(const void* data, const std::vector<size_m>& shape, dtype t);
    static matrix empty(const std::vector<size_m>& shape, dtype t);

    // frontends (lazy: build a node, compute metadata once)
    matrix sum(int axis, bool keepdims = false) const;
    matrix max(int axis, bool keepdims = false) const;
    matrix min(int axis, bool keepdims = false) const;
    matrix argmax(int axis, bool keepdims = false) const;
    matrix argmin(int axis, bool keepdims = false) const;
    matrix sum() const;  // all elements (flatten then sum(0), Matrix.mm:15215-15218)
    // axes start..end flattened into one and reduced (flatten(start, end).op(start, keepdims):
    // Matrix.mm:15210-15213, 14917-14920, 15061-15064); max() / min() over all elements (14922-14925,
    // 15066-15069)
    matrix sum(int start, int end, bool keepdims = false) const;
    matrix max(int start, int end, bool keepdims = false) const;
    matrix min(int start, int end, bool keepdims = false) const;
    matrix max() const;
    matrix min() const;
    // axes start..end merged into one (Matrix.mm:623-657): a view when they are contiguous with each
    // other, else a contiguous copy first (the reference's reshape with a new buffer)
    matrix flatten(int start_dim = 0, int end_dim = -1) const;
    matrix mean(int axis, bool keepdims = false) const;
    matrix rms(int axis, bool keepdims = false) const;
    matrix norm(int axis, bool keepdims = false) const;
    matrix mean() const;  // all elements (a contiguous matrix viewed as 1-D)
    matrix rms() const;
    matrix norm() const;
    // element type conversion; without make_contig the output keeps this matrix's strides, as the
    // promotion in front of binary ops does
    matrix astype(dtype t, bool make_contig = false) const;
    static matrix scalar(float value, dtype t);
    friend matrix operator+(const matrix& a, const matrix& b);
    friend matrix operator-(const matrix& a, const matrix& b);
    friend matrix operator*(const matrix& a, const matrix& b);
    friend matrix operator/(const matrix& a, const matrix& b);
    static matrix max(const matrix& a, const matrix& b);
    static matrix min(const matrix& a, const matrix& b);
    static matrix exp(const matrix& x);
    static matrix sqrt(const matrix& x);
    static matrix equal(const matrix& a, const matrix& b);
    static matrix greater(const matrix& a, const matrix& b);
    static matrix less(const matrix& a, const matrix& b);
    static matrix logical_and(const matrix& a, const matrix& b);
    static matrix where(const matrix& cond, const matrix& a, const matrix& b);
    static matrix floor(const matrix& x);
    static matrix full(const std::vector<size_m>& shape, const matrix& value, dtype t);
    // arctan2(a, b) / arcsin(x) on inputs cast to Float, Float output (Matrix.mm:13573-13580)
    static matrix arctan2(const matrix& a, const matrix& b);
    static matrix arcsin(const matrix& x);
    // max(0, ceil((stop - start) / step)) elements start + i * step of dtype t (Matrix.mm:13595-13604)
    static matrix arange(double start, double stop, double step = 1, dtype t = dtype::Float);
    static matrix arange(double stop, dtype t = dtype::Float) { return arange(0, stop, 1, t); }

    // views of an evaluated matrix (no copy: new strides / offset over the same buffer)
    matrix transpose(int a, int b) const;
    matrix slice(int axis, size_m start, size_m end) const;
    matrix reshape(const std::vector<size_m>& shape) const;  // contiguous, evaluated input

    // evaluation
    void eval();                // compile + execute in one pass, then synchronise
    void compile();             // allocate every output (COMPILE_TRACE), fuse the softmax trace
    void execute();             // kernels only; recorded into a CUDA graph per set of bound device
                                // pointers (first execute with them), replayed while they stay bound
    void clear_trace_checks();  // resets `evaluated` down the graph before re-running a pass
    // several roots compiled as one graph (fusions across roots: Max + ArgMax, Min + ArgMin of the same
    // input, axis and keepdims read the input once) and executed as one pass
    static void compile(const std::vector<matrix*>& roots);
    static void execute(const std::vector<matrix*>& roots);

    // Compiled functions (Matrix.mm:1076-1149): func is traced once on `sample` (a swap leaf), compiled,
    // and the returned function builds, per call, a lazy node that hands the caller's input buffer to the
    // compiled graph's input and the call's own output buffer to the graph's output, then executes the
    // graph (CompiledNodePrimitive / MultiInputCompilePrimitive, primitives.cpp:3844-4251).  Inputs must
    // have the samples' shapes, strides and dtypes.  Each call's outputs are distinct buffers.
    static std::function<matrix(const matrix&)> jit_graph_gpu(std::function<matrix(matrix)> func, matrix sample);
    static std::function<std::vector<matrix>(const std::vector<matrix>&)> multi_jit_graph_gpu(
        std::function<std::vector<matrix>(std::vector<matrix>)> func, const std::vector<matrix>& sample_inputs);

    // host access (evaluates first)
    std::vector<uint8_t> to_host_bytes() const;
    template <typename T>
    std::vector<T> to_host() const {
        std::vector<uint8_t> b = to_host_bytes();
        std::vector<T> out(b.size() / sizeof(T));
        if (!b.empty()) std::memcpy(out.data(), b.data(), b.size());
        return out;
    }
    // overwrite a leaf's contents in place (the next execute() sees the new values)
    void upload(const void* data);

    // metadata
    uint32_t dims() const { return (uint32_t)shape_.size(); }
    const std::vector<size_m>& shape() const { return shape_; }
    const std::vector<size_m>& strides() const { return strides_; }
    dtype type() const { return type_; }
    uint64_t total_size() const;
    bool has_tape() const { return (bool)tape_; }
    const Primitive* tape() const { return tape_.get(); }
    void* data() const;  // device pointer of the view's first element (nullptr before allocation)

    // used by the primitives
    void ensure_buffer(const std::shared_ptr<Buffer>& adopt);
    void rebind_buffer(const std::shared_ptr<Buffer>& b) { buffer_ = b; }
    const std::shared_ptr<Buffer>& buffer() const { return buffer_; }
    std::shared_ptr<Primitive> tape_ptr() const { return tape_; }
    void set_tape(std::shared_ptr<Primitive> p) { tape_ = std::move(p); }
    void set_layout(std::vector<size_m> shape, std::vector<size_m> strides, dtype t, uint64_t offset = 0);

private:
    std::shared_ptr<Buffer> buffer_;
    uint64_t offset_ = 0;  // elements
    std::vector<size_m> shape_, strides_;
    dtype type_ = dtype::Float;
    std::shared_ptr<Primitive> tape_;
    std::shared_ptr<GraphCache> graphs_;  // the recorded execute passes of the graph rooted here
};

// ------------------------------------------------------------------------------------------------
// Several GPUs.  The reference drives one Metal device (Mods/GPUManager.h:53-54) and has no multi-GPU
// API; this mirrors the C ABI's communicator (mtxc_comm_*, mtxc_reduce_sharded) for C++ callers.  One
// process (or host thread) per GPU, each bound with init(device); like any collective, every rank builds
// and evaluates the same sharded reductions in the same order.
// ------------------------------------------------------------------------------------------------
class Communicator {
public:
    // A new communicator id (rank 0 makes it; the caller carries it to the other ranks: MPI, a file, ...).
    static std::string unique_id();
    // Joins the calling thread as `rank` of `nranks` (mtxc_comm_init); blocks until every rank has joined.
    Communicator(int nranks, int rank, const std::string& id, size_t buffer_bytes = 0);
    // Waits for the thread's stream and releases the communicator.  Call barrier() on every rank first:
    // a rank still exchanging writes into the other ranks' buffers.
    ~Communicator();
    Communicator(const Communicator&) = delete;
    Communicator& operator=(const Communicator&) = delete;
    int size() const { return nranks_; }
    int rank() const { return rank_; }
    // whether the exchanges run as one kernel over NVLink peer memory (else NCCL all-gather + merge)
    bool peer_exchange() const;
    // waits for the thread's stream; whether an exchange since the last query gave up waiting for a rank
    bool timed_out();
    // a one-value exchange on every rank, then a wait: once it returns, no rank writes into this rank's
    // buffers for any earlier exchange
    void barrier();

private:
    int nranks_ = 1, rank_ = 0;
    void* token_ = nullptr;  // one int32 of device memory for barrier()
};

enum class ReduceOp { Sum = 0, Max = 1, Min = 2, ArgMax = 3, ArgMin = 4 };

// local.op(0, keepdims) of a matrix sharded along axis 0 across the ranks of the calling thread's
// Communicator: this rank holds `local`, a contiguous slice of the global axis (possibly empty), and
// first_rows[r] is the global index of rank r's first row (ArgMax / ArgMin turn local indices into global
// ones with it; the other ops may pass none).  Lazy like the other reductions; the result is the whole
// reduction, identical on every rank, with the reference's order and tie rules across the shards (float
// sums in rank order, the first global index of an extreme).
matrix reduce_sharded(ReduceOp op, const matrix& local, const std::vector<int64_t>& first_rows = {},
                      bool keepdims = false);

}  // namespace mtx
