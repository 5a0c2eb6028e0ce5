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
//               matrix::scalar(v, t)                                           (a 0-d matrix holding dtype_cast<t>(v))
//   primitives  allocate-or-adopt the output, return before computing under COMPILE_TRACE, run once
//               per pass (`evaluated`), then call the backend (primitives.cpp:2836-2902)
//   evaluation  eval() = compile + execute in one pass; compile() allocates every output and fuses
//               the softmax trace; execute() runs kernels only -- the first execute is recorded into a
//               CUDA graph, later ones replay it (Matrix.mm:8415-8475)
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

// Device memory owned by one or more matrices (the reference's buffer + refCount).
struct Buffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    explicit Buffer(size_t n);
    ~Buffer();
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;
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
};

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

    // views of an evaluated matrix (no copy: new strides / offset over the same buffer)
    matrix transpose(int a, int b) const;
    matrix slice(int axis, size_m start, size_m end) const;
    matrix reshape(const std::vector<size_m>& shape) const;  // contiguous, evaluated input

    // evaluation
    void eval();                // compile + execute in one pass, then synchronise
    void compile();             // allocate every output (COMPILE_TRACE), fuse the softmax trace
    void execute();             // kernels only; recorded into a CUDA graph the first time, replayed after
    void clear_trace_checks();  // resets `evaluated` down the graph before re-running a pass

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
    const std::shared_ptr<Buffer>& buffer() const { return buffer_; }
    std::shared_ptr<Primitive> tape_ptr() const { return tape_; }
    void set_tape(std::shared_ptr<Primitive> p) { tape_ = std::move(p); }
    void set_layout(std::vector<size_m> shape, std::vector<size_m> strides, dtype t, uint64_t offset = 0);

private:
    matrix flat(const char* what) const;  // flatten(0, -1) of a contiguous matrix
    std::shared_ptr<Buffer> buffer_;
    uint64_t offset_ = 0;  // elements
    std::vector<size_m> shape_, strides_;
    dtype type_ = dtype::Float;
    std::shared_ptr<Primitive> tape_;
    std::shared_ptr<void> graph_;  // the recorded execute pass of the graph rooted here
};

}  // namespace mtx
