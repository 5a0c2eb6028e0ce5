// mtx.cpp -- the C++ host mirror: graph nodes, metadata and evaluation over the C ABI.
#include "mtx.hpp"

#include <algorithm>
#include <cstring>
#include <functional>
#include <set>

#include "mtxc.h"
#include "nvtx3/nvToolsExt.h"  // header-only NVTX v3: ranges cost nothing unless a profiler is attached

namespace mtx {

namespace {

// An NVTX range over a scope (eval / compile / execute show up as named ranges in Nsight tools).
struct Range {
    explicit Range(const char* name) { nvtxRangePushA(name); }
    ~Range() { nvtxRangePop(); }
};

[[noreturn]] void raise(int rc, const std::string& where) {
    std::string msg = where + ": " + mtxc_last_error();
    if (rc == MTXC_ERR_SHAPE || rc == MTXC_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void check(int rc, const char* where) {
    if (rc != MTXC_OK) raise(rc, where);
}

std::vector<size_m> row_major(const std::vector<size_m>& shape) {
    std::vector<size_m> s(shape.size());
    size_m acc = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
        s[i] = acc;
        acc *= shape[i];
    }
    return s;
}

uint64_t product(const std::vector<size_m>& shape) {
    uint64_t p = 1;
    for (size_m e : shape) p *= e;
    return p;
}

bool contiguous(const std::vector<size_m>& shape, const std::vector<size_m>& strides) {
    uint64_t acc = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
        if (shape[i] != 1 && strides[i] != acc) return false;
        acc *= shape[i];
    }
    return true;
}

int normalize_axis(int axis, uint32_t dims) {
    if (axis < 0) axis += (int)dims;
    if (axis < 0 || axis >= (int)dims) throw std::invalid_argument("axis out of range");
    return axis;
}

// Elements a layout spans (the reference's effectiveBufferSize): the last element's offset + 1.
uint64_t span(const std::vector<size_m>& shape, const std::vector<size_m>& strides) {
    uint64_t last = 0;
    for (size_t i = 0; i < shape.size(); ++i) {
        if (shape[i] == 0) return 0;
        last += (uint64_t)(shape[i] - 1) * strides[i];
    }
    return last + 1;
}

// Allocate-or-adopt the output and fill the tape's cache (primitives.cpp:2866-2882), before the
// single COMPILE_TRACE return.
void allocate_output(Primitive& p, matrix& out) {
    if (!p.out_buffer)
        p.out_buffer = std::make_shared<Buffer>(std::max<uint64_t>(span(out.shape(), out.strides()), 1) *
                                                dtype_size(out.type()));
    out.ensure_buffer(p.out_buffer);
}

// DFS into an input that is still a graph node.
void eval_input(matrix& in, EvalType t) {
    if (in.has_tape()) {
        auto p = in.tape_ptr();
        if (!p->evaluated || t == EvalType::COMPILE_TRACE) p->eval(in, t);
        in.ensure_buffer(p->out_buffer);
    }
}

// ------------------------------------------------------------------------------------------
// Primitives
// ------------------------------------------------------------------------------------------

// Sum / Max / Min / ArgMax / ArgMin (primitives.cpp:2825-2971, 1967-2252, 7584-7799)
class ReducePrimitive : public Primitive {
public:
    ReducePrimitive(int op, const matrix& in, int axis, bool keepdims, const std::vector<size_m>& out_shape)
        : op_(op), input_(in), axis_(axis), keepdims_(keepdims) {
        // collapse_dims_reduce(shape, out.strides, in.strides, dims, axis, false, !keepdims, UINT32_MAX)
        const uint32_t dims = in.dims();
        std::vector<size_m> out_strides = row_major(out_shape);
        out_strides.resize(dims, 0);
        cdims_ = mtxc_collapse_dims_reduce2(in.shape().data(), out_strides.data(), in.strides().data(), dims, axis, 0,
                                            keepdims ? 0 : 1, 0xFFFFFFFFu, shape_, s_out_, s_in_);
        rstride_ = in.strides()[axis];
        rlen_ = in.shape()[axis];
    }
    void eval(matrix& out, EvalType t) override {
        eval_input(input_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        check(mtxc_reduce(op_, (int)input_.type(), out.data(), input_.data(), rstride_, rlen_, cdims_, shape_, s_out_,
                          s_in_),
              "mtxc_reduce");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (input_.has_tape()) input_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&input_}; }
    const char* name() const override {
        static const char* n[] = {"Sum", "MaxReduction", "MinReduction", "ArgMax", "ArgMin"};
        return n[op_];
    }
    int op() const { return op_; }
    int axis() const { return axis_; }
    bool keepdims() const { return keepdims_; }
    const matrix& input() const { return input_; }

private:
    int op_;
    matrix input_;
    int axis_;
    bool keepdims_;
    uint32_t cdims_ = 0, rstride_ = 0, rlen_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, s_out_[MTXC_MAX_DIMS] = {}, s_in_[MTXC_MAX_DIMS] = {};
};

// Add / Sub / Mul / Div / Max / Min with broadcasting (primitives.cpp:397-1046, 2515-2823)
class BinaryPrimitive : public Primitive {
public:
    BinaryPrimitive(int op, const matrix& a, const matrix& b, std::vector<size_m>& out_shape) : op_(op), a_(a), b_(b) {
        const int d1 = (int)a.dims(), d2 = (int)b.dims();
        const int od = std::max(d1, d2);
        uint32_t os[MTXC_MAX_DIMS], ost[MTXC_MAX_DIMS], ash[MTXC_MAX_DIMS], ast[MTXC_MAX_DIMS], bsh[MTXC_MAX_DIMS],
            bst[MTXC_MAX_DIMS];
        check(mtxc_broadcast_shapes(a.shape().data(), a.strides().data(), d1, b.shape().data(), b.strides().data(), d2,
                                    os, ost, ash, ast, bsh, bst),
              "broadcast_shapes");
        out_shape.assign(os, os + od);
        // collapse_dims(desc_a.shape, desc_a.strides, desc_b.strides, result.strides, dims, INT32_MAX)
        cdims_ = mtxc_collapse_dims3(ash, ast, bst, ost, (uint32_t)od, 0x7FFFFFFFu, shape_, sa_, sb_, sr_);
    }
    void eval(matrix& out, EvalType t) override {
        eval_input(a_, t);
        eval_input(b_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        if (a_.type() != b_.type())  // promotion fused into the op
            check(mtxc_broadcast_binary_mixed(op_, (int)out.type(), (int)a_.type(), (int)b_.type(), out.data(),
                                              a_.data(), b_.data(), cdims_, shape_, sr_, sa_, sb_),
                  "mtxc_broadcast_binary_mixed");
        else
            check(mtxc_broadcast_binary(op_, (int)a_.type(), out.data(), a_.data(), b_.data(), cdims_, shape_, sr_,
                                        sa_, sb_),
                  "mtxc_broadcast_binary");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (a_.has_tape()) a_.tape_ptr()->clear_trace_checks();
        if (b_.has_tape()) b_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&a_, &b_}; }
    const char* name() const override {
        static const char* n[] = {"Addition", "Subtraction", "Multiplication", "Division", "Max", "Min", "Equal"};
        return n[op_];
    }
    int op() const { return op_; }
    const matrix& a() const { return a_; }
    const matrix& b() const { return b_; }

private:
    int op_;
    matrix a_, b_;
    uint32_t cdims_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, sr_[MTXC_MAX_DIMS] = {}, sa_[MTXC_MAX_DIMS] = {}, sb_[MTXC_MAX_DIMS] = {};
};

// exp / sqrt (ExpPrimitive primitives.cpp:5332-5463, SqrtPrimitive)
class UnaryPrimitive : public Primitive {
public:
    UnaryPrimitive(int op, const matrix& in) : op_(op), input_(in) {
        std::vector<size_m> out_strides = row_major(in.shape());
        cdims_ = mtxc_collapse_dims2(in.shape().data(), out_strides.data(), in.strides().data(), in.dims(), 0x7FFFFFFFu,
                                     shape_, s_out_, s_in_);
    }
    void eval(matrix& out, EvalType t) override {
        eval_input(input_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        check(mtxc_unary(op_, (int)input_.type(), out.data(), input_.data(), cdims_, shape_, s_out_, s_in_), "mtxc_unary");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (input_.has_tape()) input_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&input_}; }
    const char* name() const override { return op_ == MTXC_UNARY_EXP ? "Exp" : "Sqrt"; }
    int op() const { return op_; }
    const matrix& input() const { return input_; }

private:
    int op_;
    matrix input_;
    uint32_t cdims_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, s_out_[MTXC_MAX_DIMS] = {}, s_in_[MTXC_MAX_DIMS] = {};
};

// astype (AsTypePrimitive, primitives.cpp:3510-3591): collapse_dims(in.shape, out.strides, in.strides)
class AsTypePrimitive : public Primitive {
public:
    AsTypePrimitive(const matrix& in, const std::vector<size_m>& out_strides) : input_(in) {
        cdims_ = mtxc_collapse_dims2(in.shape().data(), out_strides.data(), in.strides().data(), in.dims(), 0x7FFFFFFFu,
                                     shape_, s_out_, s_in_);
    }
    void eval(matrix& out, EvalType t) override {
        eval_input(input_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        check(mtxc_astype((int)out.type(), (int)input_.type(), out.data(), input_.data(), cdims_, shape_, s_out_, s_in_),
              "mtxc_astype");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (input_.has_tape()) input_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&input_}; }
    const char* name() const override { return "AsType"; }

private:
    matrix input_;
    uint32_t cdims_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, s_out_[MTXC_MAX_DIMS] = {}, s_in_[MTXC_MAX_DIMS] = {};
};

// greater / less / logical_and / where / floor / full over make_pointwise's collapse
// (Matrix.mm:13511-13556); the output is contiguous.
class PointwisePrimitive : public Primitive {
public:
    PointwisePrimitive(int op, std::vector<matrix> ins, const std::vector<size_m>& out_shape)
        : op_(op), inputs_(std::move(ins)) {
        const uint32_t rank = (uint32_t)out_shape.size();
        std::vector<size_m> rows(inputs_.size() * std::max<uint32_t>(rank, 1), 0);
        for (size_t i = 0; i < inputs_.size(); ++i) {
            const matrix& in = inputs_[i];
            for (uint32_t d = 0; d < in.dims(); ++d)
                rows[i * rank + rank - in.dims() + d] = in.shape()[d] == 1 ? 0 : in.strides()[d];
        }
        cdims_ = mtxc_pointwise_collapse(out_shape.data(), rank, rows.data(), (uint32_t)inputs_.size(), shape_, strides_);
        if (cdims_ == 0xFFFFFFFFu) throw std::invalid_argument("pointwise output exceeds the rank or 32-bit size limit");
    }
    void eval(matrix& out, EvalType t) override {
        for (matrix& in : inputs_) eval_input(in, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        if (out.total_size() == 0) return;  // the backends return before reading anything
        const void* ptrs[3] = {};
        for (size_t i = 0; i < inputs_.size(); ++i) ptrs[i] = inputs_[i].data();
        const int dt = (int)inputs_[op_ == MTXC_PW_WHERE ? 1 : 0].type();
        check(mtxc_pointwise(op_, dt, out.data(), ptrs, (uint32_t)inputs_.size(), cdims_, shape_, strides_),
              "mtxc_pointwise");
    }
    void clear_trace_checks() override {
        evaluated = false;
        for (matrix& in : inputs_)
            if (in.has_tape()) in.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override {
        std::vector<matrix*> v;
        for (matrix& in : inputs_) v.push_back(&in);
        return v;
    }
    const char* name() const override {
        static const char* n[] = {"Greater", "Less", "LogicalAnd", "Where", "Floor", "Full"};
        return n[op_];
    }

private:
    int op_;
    std::vector<matrix> inputs_;
    uint32_t cdims_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, strides_[3 * MTXC_MAX_DIMS] = {};
};

// mean / rms / norm as one node (mtxc_reduce_stat); metadata as ReducePrimitive's
class StatPrimitive : public Primitive {
public:
    StatPrimitive(int stat, const matrix& in, int axis, bool keepdims, const std::vector<size_m>& out_shape)
        : stat_(stat), input_(in) {
        const uint32_t dims = in.dims();
        std::vector<size_m> out_strides = row_major(out_shape);
        out_strides.resize(dims, 0);
        cdims_ = mtxc_collapse_dims_reduce2(in.shape().data(), out_strides.data(), in.strides().data(), dims, axis, 0,
                                            keepdims ? 0 : 1, 0xFFFFFFFFu, shape_, s_out_, s_in_);
        rstride_ = in.strides()[axis];
        rlen_ = in.shape()[axis];
    }
    void eval(matrix& out, EvalType t) override {
        eval_input(input_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        check(mtxc_reduce_stat(stat_, (int)input_.type(), out.data(), input_.data(), rstride_, rlen_, cdims_, shape_,
                               s_out_, s_in_),
              "mtxc_reduce_stat");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (input_.has_tape()) input_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&input_}; }
    const char* name() const override {
        static const char* n[] = {"Mean", "Rms", "Norm"};
        return n[stat_];
    }
    uint32_t rlen() const { return rlen_; }

private:
    int stat_;
    matrix input_;
    uint32_t cdims_ = 0, rstride_ = 0, rlen_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, s_out_[MTXC_MAX_DIMS] = {}, s_in_[MTXC_MAX_DIMS] = {};
};

// The softmax trace over the last axis, fused by compile() (no counterpart primitive in the reference)
class FusedSoftmaxPrimitive : public Primitive {
public:
    explicit FusedSoftmaxPrimitive(const matrix& x) : input_(x) {}
    void eval(matrix& out, EvalType t) override {
        eval_input(input_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        const size_m n = input_.shape().back();
        const uint64_t rows = n ? input_.total_size() / n : 0;
        check(mtxc_softmax_lastdim((int)input_.type(), out.data(), input_.data(), rows, n, n, n), "mtxc_softmax_lastdim");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (input_.has_tape()) input_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&input_}; }
    const char* name() const override { return "FusedSoftmax"; }

private:
    matrix input_;
};

// Recognises y = e / e.sum(-1, true) with e = exp(x - x.max(-1, true)) on contiguous float rows the
// fused kernel accepts, and returns the fused node (or nullptr).
std::shared_ptr<Primitive> match_softmax(const matrix& y) {
    auto* div = dynamic_cast<const BinaryPrimitive*>(y.tape());
    if (!div || div->op() != MTXC_BINARY_DIV) return nullptr;
    auto* s = dynamic_cast<const ReducePrimitive*>(div->b().tape());
    if (!s || s->op() != MTXC_REDUCE_SUM || !s->keepdims() || s->input().tape() != div->a().tape()) return nullptr;
    auto* e = dynamic_cast<const UnaryPrimitive*>(div->a().tape());
    if (!e || e->op() != MTXC_UNARY_EXP) return nullptr;
    auto* t = dynamic_cast<const BinaryPrimitive*>(e->input().tape());
    if (!t || t->op() != MTXC_BINARY_SUB) return nullptr;
    auto* m = dynamic_cast<const ReducePrimitive*>(t->b().tape());
    if (!m || m->op() != MTXC_REDUCE_MAX || !m->keepdims()) return nullptr;
    const matrix& x = t->a();
    const matrix& xm = m->input();
    const bool same_x = x.tape() ? x.tape() == xm.tape() : (x.buffer() && x.buffer() == xm.buffer() &&
                                                            x.data() == xm.data() && x.strides() == xm.strides());
    if (!same_x || x.type() != dtype::Float || x.dims() == 0) return nullptr;
    const int last = (int)x.dims() - 1;
    if (s->axis() != last || m->axis() != last || !contiguous(x.shape(), x.strides())) return nullptr;
    if (x.shape() != y.shape() || x.shape()[last] % 4 != 0 || x.shape()[last] > MTXC_SOFTMAX_MAX_ROW) return nullptr;
    return std::make_shared<FusedSoftmaxPrimitive>(x);
}

void fuse_graph(matrix& root) {
    std::set<const Primitive*> seen;
    std::function<void(matrix&)> visit = [&](matrix& m) {
        if (!m.has_tape()) return;
        if (auto fused = match_softmax(m)) m.set_tape(fused);
        Primitive* p = m.tape_ptr().get();
        if (!seen.insert(p).second) return;
        for (matrix* in : p->inputs()) visit(*in);
    };
    visit(root);
}

matrix make_reduce(int op, const matrix& x, int axis, bool keepdims) {
    if (x.dims() == 0) throw std::invalid_argument("reduction of a 0-d matrix");
    axis = normalize_axis(axis, x.dims());
    std::vector<size_m> out_shape = x.shape();
    if (keepdims) out_shape[axis] = 1;
    else out_shape.erase(out_shape.begin() + axis);
    const bool arg = op == MTXC_REDUCE_ARGMAX || op == MTXC_REDUCE_ARGMIN;
    matrix out;
    out.set_layout(out_shape, row_major(out_shape), arg ? dtype::Int32 : x.type());
    out.set_tape(std::make_shared<ReducePrimitive>(op, x, axis, keepdims, out_shape));
    return out;
}

matrix make_binary(int op, const matrix& a, const matrix& b) {
    // + - * / and equal promote both operands with astype first (Matrix.mm:8313-8315, 14452-14454).
    // max / min(a, b) promote only the result dtype and read b's memory as a's type (Matrix.mm:13364-13366,
    // 13459), which is meaningful only for equal dtypes; mixed dtypes are refused there.
    const bool promotes = op != MTXC_BINARY_MAX && op != MTXC_BINARY_MIN;
    if (!promotes && a.type() != b.type())
        throw std::runtime_error("max / min(a, b) of mixed dtypes: cast one operand with astype first");
    const dtype common = promote_types(a.type(), b.type());
    // the conversion of both operands happens inside the op's kernel (mtxc_broadcast_binary_mixed), same
    // bits as astype + op without the promoted copies
    const bool fused = promotes && a.type() != b.type() && common != dtype::Complex64;
    const matrix lhs = (a.type() == common || fused) ? a : a.astype(common);
    const matrix rhs = (b.type() == common || fused) ? b : b.astype(common);
    std::vector<size_m> out_shape;
    auto prim = std::make_shared<BinaryPrimitive>(op, lhs, rhs, out_shape);
    matrix out;
    out.set_layout(out_shape, row_major(out_shape), common);
    out.set_tape(prim);
    return out;
}

// pointwise_cast / pointwise_shape / make_pointwise (Matrix.mm:13487-13556)
matrix pointwise_cast(const matrix& x, dtype t) { return x.type() == t ? x : x.astype(t); }

std::vector<size_m> pointwise_shape(const std::vector<matrix>& ins) {
    uint32_t rank = 0;
    for (const matrix& in : ins) rank = std::max(rank, in.dims());
    if (rank > MTXC_MAX_DIMS) throw std::invalid_argument("pointwise rank exceeds MAX_TENSOR_DIMS");
    std::vector<size_m> shape(rank, 1);
    for (const matrix& in : ins)
        for (uint32_t d = 0; d < in.dims(); ++d) {
            size_m& n = shape[rank - in.dims() + d];
            const size_m m = in.shape()[d];
            if (n == 1) n = m;
            else if (m != 1 && n != m) throw std::invalid_argument("incompatible pointwise broadcast shapes");
        }
    return shape;
}

matrix make_pointwise(int op, const std::vector<matrix>& ins, const std::vector<size_m>& shape, dtype t) {
    for (const matrix& in : ins) {
        if (in.dims() > shape.size()) throw std::invalid_argument("input rank exceeds pointwise output rank");
        for (uint32_t d = 0; d < in.dims(); ++d)
            if (in.shape()[d] != 1 && in.shape()[d] != shape[shape.size() - in.dims() + d])
                throw std::invalid_argument("input cannot broadcast to pointwise output shape");
    }
    auto prim = std::make_shared<PointwisePrimitive>(op, ins, shape);
    matrix out;
    out.set_layout(shape, row_major(shape), t);
    out.set_tape(prim);
    return out;
}

matrix make_stat(int stat, const matrix& x, int axis, bool keepdims) {
    if (x.dims() == 0) throw std::invalid_argument("reduction of a 0-d matrix");
    axis = normalize_axis(axis, x.dims());
    std::vector<size_m> out_shape = x.shape();
    if (keepdims) out_shape[axis] = 1;
    else out_shape.erase(out_shape.begin() + axis);
    const int oc = mtxc_reduce_stat_dtype(stat, (int)x.type(), x.shape()[axis]);
    if (oc < 0) throw std::runtime_error("mean / rms / norm: unsupported dtype");
    matrix out;
    out.set_layout(out_shape, row_major(out_shape), (dtype)oc);
    out.set_tape(std::make_shared<StatPrimitive>(stat, x, axis, keepdims, out_shape));
    return out;
}


}  // namespace

// ------------------------------------------------------------------------------------------
// dtype helpers, runtime
// ------------------------------------------------------------------------------------------
size_t dtype_size(dtype t) {
    static const size_t sizes[] = {4, 2, 1, 4, 2, 4, 2, 1, 1, 8, 2, 8, 8};
    return sizes[(int)t];
}

dtype promote_types(dtype a, dtype b) { return (dtype)mtxc_promote_types((int)a, (int)b); }

void init(int device) { check(mtxc_init(device), "mtxc_init"); }

Buffer::Buffer(size_t n) : bytes(n) { check(mtxc_alloc(n, &ptr), "mtxc_alloc"); }
Buffer::~Buffer() { mtxc_free(ptr); }

// ------------------------------------------------------------------------------------------
// matrix
// ------------------------------------------------------------------------------------------
uint64_t matrix::total_size() const { return product(shape_); }

void matrix::set_layout(std::vector<size_m> shape, std::vector<size_m> strides, dtype t, uint64_t offset) {
    if (shape.size() > MTXC_MAX_DIMS) throw std::invalid_argument("rank above MTXC_MAX_DIMS");
    shape_ = std::move(shape);
    strides_ = std::move(strides);
    type_ = t;
    offset_ = offset;
}

void matrix::ensure_buffer(const std::shared_ptr<Buffer>& adopt) {
    if (!buffer_) buffer_ = adopt;
}

void* matrix::data() const {
    const Buffer* b = buffer_ ? buffer_.get() : (tape_ ? tape_->out_buffer.get() : nullptr);
    if (!b) return nullptr;
    return static_cast<uint8_t*>(b->ptr) + offset_ * dtype_size(type_);
}

matrix matrix::empty(const std::vector<size_m>& shape, dtype t) {
    matrix m;
    m.set_layout(shape, row_major(shape), t);
    m.buffer_ = std::make_shared<Buffer>(m.total_size() * dtype_size(t));
    return m;
}

matrix matrix::from_host(const void* data, const std::vector<size_m>& shape, dtype t) {
    matrix m = empty(shape, t);
    m.upload(data);
    return m;
}

void matrix::upload(const void* data) {
    if (tape_) throw std::runtime_error("upload: only leaves hold caller data");
    if (!contiguous(shape_, strides_)) throw std::runtime_error("upload: not contiguous");
    check(mtxc_upload(this->data(), data, total_size() * dtype_size(type_)), "mtxc_upload");
    check(mtxc_sync(), "mtxc_sync");
}

matrix matrix::sum(int axis, bool keepdims) const { return make_reduce(MTXC_REDUCE_SUM, *this, axis, keepdims); }
matrix matrix::max(int axis, bool keepdims) const { return make_reduce(MTXC_REDUCE_MAX, *this, axis, keepdims); }
matrix matrix::min(int axis, bool keepdims) const { return make_reduce(MTXC_REDUCE_MIN, *this, axis, keepdims); }
matrix matrix::argmax(int axis, bool keepdims) const { return make_reduce(MTXC_REDUCE_ARGMAX, *this, axis, keepdims); }
matrix matrix::argmin(int axis, bool keepdims) const { return make_reduce(MTXC_REDUCE_ARGMIN, *this, axis, keepdims); }

matrix matrix::sum() const { return flat("sum()").sum(0); }

matrix operator+(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_ADD, a, b); }
matrix operator-(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_SUB, a, b); }
matrix operator*(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_MUL, a, b); }
matrix operator/(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_DIV, a, b); }
matrix matrix::max(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_MAX, a, b); }
matrix matrix::min(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_MIN, a, b); }

namespace {
// exp / sqrt promote their input to promote_types(type, Float16) (Matrix.mm:6798-6811, 6934-6947)
matrix make_unary(int op, const matrix& x) {
    const dtype t = promote_types(x.type(), dtype::Float16);
    if (t != dtype::Float && t != dtype::Float16) throw std::runtime_error("exp / sqrt: unsupported dtype");
    const matrix in = x.type() == t ? x : x.astype(t, true);
    matrix out;
    out.set_layout(in.shape(), row_major(in.shape()), t);
    out.set_tape(std::make_shared<UnaryPrimitive>(op, in));
    return out;
}
}  // namespace

matrix matrix::exp(const matrix& x) { return make_unary(MTXC_UNARY_EXP, x); }
matrix matrix::sqrt(const matrix& x) { return make_unary(MTXC_UNARY_SQRT, x); }
matrix matrix::equal(const matrix& a, const matrix& b) { return make_binary(MTXC_BINARY_EQUAL, a, b); }

matrix matrix::astype(dtype t, bool make_contig) const {
    std::vector<size_m> out_strides = make_contig ? row_major(shape_) : strides_;
    matrix out;
    out.set_layout(shape_, out_strides, t);
    out.set_tape(std::make_shared<AsTypePrimitive>(*this, out_strides));
    return out;
}

matrix matrix::scalar(float value, dtype t) {
    // matrix::scalar(value, t) holds dtype_cast<t>(value): converted once, on the device
    matrix f = from_host(&value, {}, dtype::Float);
    if (t == dtype::Float) return f;
    matrix m = f.astype(t, true);
    m.eval();
    m.ensure_buffer(m.tape_->out_buffer);
    m.tape_.reset();
    return m;
}

matrix matrix::greater(const matrix& a, const matrix& b) {
    const dtype t = promote_types(a.type(), b.type());
    std::vector<matrix> ins{pointwise_cast(a, t), pointwise_cast(b, t)};
    return make_pointwise(MTXC_PW_GREATER, ins, pointwise_shape(ins), dtype::Bool);
}
matrix matrix::less(const matrix& a, const matrix& b) {
    const dtype t = promote_types(a.type(), b.type());
    std::vector<matrix> ins{pointwise_cast(a, t), pointwise_cast(b, t)};
    return make_pointwise(MTXC_PW_LESS, ins, pointwise_shape(ins), dtype::Bool);
}
matrix matrix::logical_and(const matrix& a, const matrix& b) {
    std::vector<matrix> ins{pointwise_cast(a, dtype::Bool), pointwise_cast(b, dtype::Bool)};
    return make_pointwise(MTXC_PW_LOGICAL_AND, ins, pointwise_shape(ins), dtype::Bool);
}
matrix matrix::where(const matrix& cond, const matrix& a, const matrix& b) {
    const dtype t = promote_types(a.type(), b.type());
    std::vector<matrix> ins{pointwise_cast(cond, dtype::Bool), pointwise_cast(a, t), pointwise_cast(b, t)};
    return make_pointwise(MTXC_PW_WHERE, ins, pointwise_shape(ins), t);
}
matrix matrix::floor(const matrix& x) { return make_pointwise(MTXC_PW_FLOOR, {x}, x.shape(), x.type()); }
matrix matrix::full(const std::vector<size_m>& shape, const matrix& value, dtype t) {
    uint64_t count = 1;
    for (size_m n : shape) {
        if (n && count > 0xFFFFFFFFull / n) throw std::overflow_error("pointwise tensor exceeds 32-bit indexing");
        count *= n;
    }
    return make_pointwise(MTXC_PW_FULL, {pointwise_cast(value, t)}, shape, t);
}

matrix matrix::mean(int axis, bool keepdims) const { return make_stat(MTXC_STAT_MEAN, *this, axis, keepdims); }
matrix matrix::rms(int axis, bool keepdims) const { return make_stat(MTXC_STAT_RMS, *this, axis, keepdims); }
matrix matrix::norm(int axis, bool keepdims) const { return make_stat(MTXC_STAT_NORM, *this, axis, keepdims); }
matrix matrix::flat(const char* what) const {
    // flatten(0, -1): a contiguous (or lazy, hence contiguous) matrix viewed as 1-D
    if (!contiguous(shape_, strides_)) throw std::runtime_error(std::string(what) + ": flatten needs a contiguous matrix");
    const uint64_t n = total_size();
    if (n > 0xFFFFFFFFull) throw std::invalid_argument(std::string(what) + ": more elements than size_m can count");
    matrix f = *this;
    f.set_layout({(size_m)n}, {1}, type_, offset_);
    return f;
}
matrix matrix::mean() const { return flat("mean()").mean(0); }
matrix matrix::rms() const { return flat("rms()").rms(0); }
matrix matrix::norm() const { return flat("norm()").norm(0); }

namespace {
matrix evaluated_view_source(const matrix& m) {
    matrix src = m;
    if (src.has_tape()) {
        if (!src.tape()->evaluated) src.eval();
        src.ensure_buffer(src.tape_ptr()->out_buffer);
    }
    return src;
}
}  // namespace

matrix matrix::transpose(int a, int b) const {
    matrix v = evaluated_view_source(*this);
    a = normalize_axis(a, dims());
    b = normalize_axis(b, dims());
    std::vector<size_m> sh = v.shape_, st = v.strides_;
    std::swap(sh[a], sh[b]);
    std::swap(st[a], st[b]);
    v.set_layout(sh, st, v.type_, v.offset_);
    v.tape_.reset();
    return v;
}

matrix matrix::slice(int axis, size_m start, size_m end) const {
    matrix v = evaluated_view_source(*this);
    axis = normalize_axis(axis, dims());
    if (start > end || end > v.shape_[axis]) throw std::invalid_argument("slice out of range");
    std::vector<size_m> sh = v.shape_;
    sh[axis] = end - start;
    v.set_layout(sh, v.strides_, v.type_, v.offset_ + (uint64_t)start * v.strides_[axis]);
    v.tape_.reset();
    return v;
}

matrix matrix::reshape(const std::vector<size_m>& shape) const {
    matrix v = evaluated_view_source(*this);
    if (!contiguous(v.shape_, v.strides_) || product(shape) != v.total_size())
        throw std::invalid_argument("reshape: needs a contiguous matrix of the same size");
    v.set_layout(shape, row_major(shape), v.type_, v.offset_);
    v.tape_.reset();
    return v;
}

void matrix::eval() {
    Range range("mtx::eval");
    if (!tape_) return;
    if (tape_->evaluated) {
        ensure_buffer(tape_->out_buffer);
        return;
    }
    tape_->eval(*this, EvalType::EVAL_INSTANTLY);
    ensure_buffer(tape_->out_buffer);
    check(mtxc_sync(), "mtxc_sync");
}

void matrix::compile() {
    Range range("mtx::compile");
    if (!tape_) return;
    fuse_graph(*this);
    tape_->eval(*this, EvalType::COMPILE_TRACE);
    ensure_buffer(tape_->out_buffer);
    graph_.reset();
}

void matrix::execute() {
    Range range("mtx::execute");
    if (!tape_) return;
    if (!tape_->out_buffer) compile();
    if (!graph_) {
        tape_->clear_trace_checks();
        check(mtxc_graph_begin(), "mtxc_graph_begin");
        try {
            tape_->eval(*this, EvalType::EXEC_TRACE);
        } catch (...) {
            void* g = nullptr;
            mtxc_graph_end(&g);
            if (g) mtxc_graph_destroy(g);
            throw;
        }
        void* g = nullptr;
        check(mtxc_graph_end(&g), "mtxc_graph_end");
        graph_ = std::shared_ptr<void>(g, [](void* p) { mtxc_graph_destroy(p); });
    }
    check(mtxc_graph_launch(graph_.get()), "mtxc_graph_launch");
    check(mtxc_sync(), "mtxc_sync");
}

void matrix::clear_trace_checks() {
    if (tape_) tape_->clear_trace_checks();
}

std::vector<uint8_t> matrix::to_host_bytes() const {
    matrix m = *this;
    if (m.tape_ && !m.tape_->evaluated && !m.graph_) m.eval();
    if (m.tape_) m.ensure_buffer(m.tape_->out_buffer);
    const size_t es = dtype_size(type_);
    std::vector<uint8_t> out(total_size() * es);
    if (out.empty()) return out;
    if (contiguous(shape_, strides_)) {
        check(mtxc_download(out.data(), m.data(), out.size()), "mtxc_download");
        check(mtxc_sync(), "mtxc_sync");
        return out;
    }
    // a strided view: fetch its span and gather on the host
    uint64_t span = 1;
    for (size_t i = 0; i < shape_.size(); ++i) span += (uint64_t)(shape_[i] - 1) * strides_[i];
    std::vector<uint8_t> raw(span * es);
    check(mtxc_download(raw.data(), m.data(), raw.size()), "mtxc_download");
    check(mtxc_sync(), "mtxc_sync");
    const uint64_t n = total_size();
    for (uint64_t g = 0; g < n; ++g) {
        uint64_t rem = g, off = 0;
        for (int i = (int)shape_.size() - 1; i >= 0; --i) {
            off += (rem % shape_[i]) * strides_[i];
            rem /= shape_[i];
        }
        std::memcpy(&out[g * es], &raw[off * es], es);
    }
    return out;
}

}  // namespace mtx
