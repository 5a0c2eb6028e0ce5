// mtx.cpp -- the C++ host mirror: graph nodes, metadata and evaluation over the C ABI.
#include "mtx.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
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

// Bytes of device memory a node's output needs.
size_t output_bytes(const matrix& out) {
    return std::max<uint64_t>(span(out.shape(), out.strides()), 1) * dtype_size(out.type());
}

// Allocate-or-adopt the output and fill the tape's cache (primitives.cpp:2866-2882), before the
// single COMPILE_TRACE return.  The handle always takes the tape's current buffer: a compiled
// function rebinds a graph's output to each call's own buffer.
void allocate_output(Primitive& p, matrix& out) {
    if (!p.out_buffer) p.out_buffer = std::make_shared<Buffer>(output_bytes(out));
    out.rebind_buffer(p.out_buffer);
}

// DFS into an input that is still a graph node; the handle follows the node's current buffer.
void eval_input(matrix& in, EvalType t) {
    if (in.has_tape()) {
        auto p = in.tape_ptr();
        if (!p->evaluated || t == EvalType::COMPILE_TRACE) p->eval(in, t);
        in.rebind_buffer(p->out_buffer);
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
    void metadata(uint32_t& cdims, uint32_t& rstride, uint32_t& rlen, uint32_t* shape, uint32_t* s_out,
                  uint32_t* s_in) const {
        cdims = cdims_;
        rstride = rstride_;
        rlen = rlen_;
        std::memcpy(shape, shape_, sizeof(shape_));
        std::memcpy(s_out, s_out_, sizeof(s_out_));
        std::memcpy(s_in, s_in_, sizeof(s_in_));
    }

private:
    int op_;
    matrix input_;
    int axis_;
    bool keepdims_;
    uint32_t cdims_ = 0, rstride_ = 0, rlen_ = 0;
    uint32_t shape_[MTXC_MAX_DIMS] = {}, s_out_[MTXC_MAX_DIMS] = {}, s_in_[MTXC_MAX_DIMS] = {};
};

// A reduction over axis 0 of a matrix sharded along that axis across the calling thread's communicator's
// ranks: the local reduction and the exchange of the partials, one mtxc_reduce_sharded call (no
// counterpart in the reference, which runs on one device).
class ShardedReducePrimitive : public Primitive {
public:
    ShardedReducePrimitive(int op, const matrix& in, bool keepdims, const std::vector<size_m>& out_shape,
                           std::vector<int64_t> first_rows)
        : op_(op), input_(in), first_rows_(std::move(first_rows)) {
        const uint32_t dims = in.dims();
        std::vector<size_m> out_strides = row_major(out_shape);
        out_strides.resize(dims, 0);
        cdims_ = mtxc_collapse_dims_reduce2(in.shape().data(), out_strides.data(), in.strides().data(), dims, 0, 0,
                                            keepdims ? 0 : 1, 0xFFFFFFFFu, shape_, s_out_, s_in_);
        rstride_ = in.strides()[0];
        rlen_ = in.shape()[0];
    }
    void eval(matrix& out, EvalType t) override {
        eval_input(input_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        const bool arg = op_ == MTXC_REDUCE_ARGMAX || op_ == MTXC_REDUCE_ARGMIN;
        check(mtxc_reduce_sharded(op_, (int)input_.type(), out.data(), input_.data(), rstride_, rlen_, cdims_, shape_,
                                  s_out_, s_in_, arg ? first_rows_.data() : nullptr),
              "mtxc_reduce_sharded");
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (input_.has_tape()) input_.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&input_}; }
    const char* name() const override {
        static const char* n[] = {"ShardedSum", "ShardedMax", "ShardedMin", "ShardedArgMax", "ShardedArgMin"};
        return n[op_];
    }

private:
    int op_;
    matrix input_;
    std::vector<int64_t> first_rows_;
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

// Max and ArgMax (or Min and ArgMin) of one input, axis and keepdims, evaluated from a single read
// (mtxc_reduce_pair) when compile() sees both among the roots it compiles together.  The two outputs stay
// separate nodes (PairOutPrimitive: the value side and the index side) that share this launch.
class PairOutPrimitive;
struct ReducePair {
    int op = MTXC_REDUCE_MAX;  // MAX or MIN
    matrix input;
    uint32_t cdims = 0, rstride = 0, rlen = 0;
    uint32_t shape[MTXC_MAX_DIMS] = {}, s_out[MTXC_MAX_DIMS] = {}, s_in[MTXC_MAX_DIMS] = {};
    std::weak_ptr<PairOutPrimitive> side[2];  // [0] values, [1] indices
    size_t side_bytes[2] = {0, 0};
    std::shared_ptr<Buffer> spare[2];         // for a side whose node no longer exists
    void prepare();                           // allocates what run() writes
    void run();
};

class PairOutPrimitive : public Primitive {
public:
    PairOutPrimitive(std::shared_ptr<ReducePair> pair, int side) : pair_(std::move(pair)), side_(side) {}
    void eval(matrix& out, EvalType t) override {
        eval_input(pair_->input, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) {
            pair_->prepare();  // both sides' buffers exist before any recorded pass
            return;
        }
        if (evaluated) return;
        pair_->run();
    }
    void clear_trace_checks() override {
        evaluated = false;
        if (pair_->input.has_tape()) pair_->input.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override { return {&pair_->input}; }
    const char* name() const override {
        static const char* n[2][2] = {{"PairMax", "PairArgMax"}, {"PairMin", "PairArgMin"}};
        return n[pair_->op == MTXC_REDUCE_MAX ? 0 : 1][side_];
    }
    void extra_bindings(std::vector<const void*>& sig) const override {
        if (auto other = pair_->side[1 - side_].lock()) sig.push_back(other->out_buffer ? other->out_buffer->ptr : nullptr);
    }

private:
    std::shared_ptr<ReducePair> pair_;
    int side_;
};

void ReducePair::prepare() {
    for (int k = 0; k < 2; ++k) {
        auto n = side[k].lock();
        if (n && !n->out_buffer) n->out_buffer = std::make_shared<Buffer>(side_bytes[k]);
        if (!n && !spare[k]) spare[k] = std::make_shared<Buffer>(side_bytes[k]);
    }
}

void ReducePair::run() {
    prepare();
    void* ptrs[2];
    std::shared_ptr<PairOutPrimitive> nodes[2];
    for (int k = 0; k < 2; ++k) {
        nodes[k] = side[k].lock();
        ptrs[k] = nodes[k] ? nodes[k]->out_buffer->ptr : spare[k]->ptr;
    }
    check(mtxc_reduce_pair(op, (int)input.type(), ptrs[0], static_cast<int32_t*>(ptrs[1]), input.data(), rstride, rlen,
                           cdims, shape, s_out, s_in),
          "mtxc_reduce_pair");
    for (auto& n : nodes)
        if (n) n->evaluated = true;
}

bool same_source(const matrix& a, const matrix& b) {
    if (a.tape() || b.tape()) return a.tape() == b.tape();
    return a.buffer() && a.buffer() == b.buffer() && a.data() == b.data() && a.shape() == b.shape() &&
           a.strides() == b.strides() && a.type() == b.type();
}

// Roots r1 = x.max(axis, k) and r2 = x.argmax(axis, k) (or min / argmin) become the two sides of one
// ReducePair.
void fuse_pairs(const std::vector<matrix*>& roots) {
    for (size_t i = 0; i < roots.size(); ++i) {
        auto* v = dynamic_cast<const ReducePrimitive*>(roots[i]->tape());
        if (!v || (v->op() != MTXC_REDUCE_MAX && v->op() != MTXC_REDUCE_MIN)) continue;
        const int want = v->op() == MTXC_REDUCE_MAX ? MTXC_REDUCE_ARGMAX : MTXC_REDUCE_ARGMIN;
        for (size_t j = 0; j < roots.size(); ++j) {
            auto* a = dynamic_cast<const ReducePrimitive*>(roots[j]->tape());
            if (!a || a->op() != want || a->axis() != v->axis() || a->keepdims() != v->keepdims() ||
                !same_source(a->input(), v->input()))
                continue;
            auto pair = std::make_shared<ReducePair>();
            pair->op = v->op();
            pair->input = v->input();
            v->metadata(pair->cdims, pair->rstride, pair->rlen, pair->shape, pair->s_out, pair->s_in);
            auto vs = std::make_shared<PairOutPrimitive>(pair, 0);
            auto is = std::make_shared<PairOutPrimitive>(pair, 1);
            pair->side[0] = vs;
            pair->side[1] = is;
            pair->side_bytes[0] = output_bytes(*roots[i]);
            pair->side_bytes[1] = output_bytes(*roots[j]);
            roots[i]->set_tape(vs);
            roots[j]->set_tape(is);
            roots[i]->rebind_buffer(nullptr);
            roots[j]->rebind_buffer(nullptr);
            break;
        }
    }
}

void fuse_graph(const std::vector<matrix*>& roots) {
    fuse_pairs(roots);
    std::set<const Primitive*> seen;
    std::function<void(matrix&)> visit = [&](matrix& m) {
        if (!m.has_tape()) return;
        if (auto fused = match_softmax(m)) m.set_tape(fused);
        Primitive* p = m.tape_ptr().get();
        if (!seen.insert(p).second) return;
        for (matrix* in : p->inputs()) visit(*in);
    };
    for (matrix* r : roots) visit(*r);
}

// A compiled function's input (the reference's SwapLeafPrimitive): a leaf whose memory is bound per call
// (out_buffer: an alias of the caller's input).  It never counts as evaluated, so every consumer's handle
// follows the current binding.
class SwapLeafPrimitive : public Primitive {
public:
    void eval(matrix& out, EvalType) override {
        if (!out_buffer) throw std::runtime_error("compiled graph: input is not bound");
        out.rebind_buffer(out_buffer);
    }
    void clear_trace_checks() override {}
    std::vector<matrix*> inputs() override { return {}; }
    const char* name() const override { return "SwapLeaf"; }
};

// arange's generator (ArangePrimitive; backend Matrix.mm:14167-14180, 14407): two one-element inputs
class ArangePrimitive : public Primitive {
public:
    ArangePrimitive(const matrix& start, const matrix& step) : start_(start), step_(step) {}
    void eval(matrix& out, EvalType t) override {
        eval_input(start_, t);
        eval_input(step_, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) return;
        if (evaluated) return;
        evaluated = true;
        check(mtxc_arange((int)out.type(), out.data(), start_.data(), step_.data(), out.total_size()), "mtxc_arange");
    }
    void clear_trace_checks() override { evaluated = false; }
    std::vector<matrix*> inputs() override { return {&start_, &step_}; }
    const char* name() const override { return "Arange"; }

private:
    matrix start_, step_;
};

void require_pointwise_real(dtype t) {
    if (t == dtype::Complex64 || (unsigned)t > (unsigned)dtype::UInt64)
        throw std::invalid_argument("pointwise operation requires a real dtype");
}

// matrix::scalar<double>(v, t): one element holding static_cast<T>(v) (dtype_cast, matrix.h:260-267)
matrix scalar_from_double(double v, dtype t) {
    uint8_t bytes[8] = {};
    switch (t) {
        case dtype::Float: { float x = (float)v; std::memcpy(bytes, &x, 4); break; }
        case dtype::Float16: { _Float16 x = (_Float16)v; std::memcpy(bytes, &x, 2); break; }
        case dtype::BFloat16: { __bf16 x = (__bf16)v; std::memcpy(bytes, &x, 2); break; }
        case dtype::UInt8: { uint8_t x = (uint8_t)v; std::memcpy(bytes, &x, 1); break; }
        case dtype::Int8: { int8_t x = (int8_t)v; std::memcpy(bytes, &x, 1); break; }
        case dtype::Int16: { int16_t x = (int16_t)v; std::memcpy(bytes, &x, 2); break; }
        case dtype::UInt16: { uint16_t x = (uint16_t)v; std::memcpy(bytes, &x, 2); break; }
        case dtype::Int32: { int32_t x = (int32_t)v; std::memcpy(bytes, &x, 4); break; }
        case dtype::UInt32: { uint32_t x = (uint32_t)v; std::memcpy(bytes, &x, 4); break; }
        case dtype::Int64: { int64_t x = (int64_t)v; std::memcpy(bytes, &x, 8); break; }
        case dtype::UInt64: { uint64_t x = (uint64_t)v; std::memcpy(bytes, &x, 8); break; }
        case dtype::Bool: { bytes[0] = v != 0.0; break; }
        default: throw std::invalid_argument("scalar: unsupported dtype");
    }
    return matrix::from_host(bytes, {}, t);
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

namespace {
// While a pass is being recorded no device memory may be freed (cudaFree would invalidate the capture):
// buffers released then -- a graph output rebound to a call's own buffer drops its previous one -- are
// freed once the recording has ended.
thread_local bool t_defer_frees = false;
thread_local std::vector<void*> t_deferred_frees;

void release_deferred() {
    std::vector<void*> v;
    v.swap(t_deferred_frees);
    for (void* p : v) mtxc_free(p);
}
}  // namespace

Buffer::Buffer(size_t n) : bytes(n) { check(mtxc_alloc(n, &ptr), "mtxc_alloc"); }
Buffer::Buffer(void* alias, size_t n, std::shared_ptr<Buffer> owner) : ptr(alias), bytes(n), owner_(std::move(owner)) {}
Buffer::~Buffer() {
    if (owner_) return;
    if (t_defer_frees) t_deferred_frees.push_back(ptr);
    else mtxc_free(ptr);
}

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

matrix matrix::sum() const { return flatten(0, -1).sum(0); }

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
matrix matrix::mean() const { return flatten(0, -1).mean(0); }
matrix matrix::rms() const { return flatten(0, -1).rms(0); }
matrix matrix::norm() const { return flatten(0, -1).norm(0); }

matrix matrix::sum(int start, int end, bool keepdims) const { return flatten(start, end).sum(start, keepdims); }
matrix matrix::max(int start, int end, bool keepdims) const { return flatten(start, end).max(start, keepdims); }
matrix matrix::min(int start, int end, bool keepdims) const { return flatten(start, end).min(start, keepdims); }
matrix matrix::max() const { return flatten(0, -1).max(0); }
matrix matrix::min() const { return flatten(0, -1).min(0); }

matrix matrix::arctan2(const matrix& a, const matrix& b) {
    require_pointwise_real(a.type());
    require_pointwise_real(b.type());
    std::vector<matrix> ins{pointwise_cast(a, dtype::Float), pointwise_cast(b, dtype::Float)};
    return make_pointwise(MTXC_PW_ARCTAN2, ins, pointwise_shape(ins), dtype::Float);
}
matrix matrix::arcsin(const matrix& x) {
    require_pointwise_real(x.type());
    return make_pointwise(MTXC_PW_ARCSIN, {pointwise_cast(x, dtype::Float)}, x.shape(), dtype::Float);
}
matrix matrix::arange(double start, double stop, double step, dtype t) {
    require_pointwise_real(t);
    if (t == dtype::Bool) throw std::invalid_argument("arange does not support Bool");
    if (!std::isfinite(start) || !std::isfinite(stop) || !std::isfinite(step) || step == 0)
        throw std::invalid_argument("arange requires finite bounds and a finite nonzero step");
    const double length = std::max(0.0, std::ceil((stop - start) / step));
    if (!std::isfinite(length) || length > 4294967295.0) throw std::overflow_error("arange exceeds 32-bit indexing");
    const size_m n = (size_m)length;
    matrix out;
    out.set_layout({n}, {1}, t);
    out.set_tape(std::make_shared<ArangePrimitive>(scalar_from_double(start, t), scalar_from_double(step, t)));
    return out;
}

matrix matrix::flatten(int start, int end) const {
    const int d = (int)dims();
    if (d == 0) {
        matrix f = *this;
        f.set_layout({1}, {1}, type_, offset_);
        return f;
    }
    if (end < 0) end += d;
    if (start < 0) start += d;
    if (start < 0 || end >= d || start > end) throw std::invalid_argument("flatten: axes out of range");
    // the range's non-unit axes must chain (each steps by the extent of the next) to merge as a view; the
    // last of them gives the merged stride
    uint64_t merged = 1;
    std::vector<int> real;
    for (int i = start; i <= end; ++i) {
        merged *= shape_[i];
        if (shape_[i] != 1) real.push_back(i);
    }
    if (merged > 0xFFFFFFFFull) throw std::invalid_argument("flatten: more elements than size_m can count");
    bool adjacent = true;
    for (size_t k = 0; k + 1 < real.size(); ++k)
        if ((uint64_t)strides_[real[k]] != (uint64_t)strides_[real[k + 1]] * shape_[real[k + 1]]) adjacent = false;
    if (merged == 0) adjacent = true;
    if (!adjacent) {  // the reference's reshape with a new buffer: a contiguous copy first
        matrix c = astype(type_, true);
        return c.flatten(start, end);
    }
    const size_m stride = real.empty() ? 1 : strides_[real.back()];
    std::vector<size_m> sh, st;
    for (int i = 0; i < start; ++i) {
        sh.push_back(shape_[i]);
        st.push_back(strides_[i]);
    }
    sh.push_back((size_m)merged);
    st.push_back(stride);
    for (int i = end + 1; i < d; ++i) {
        sh.push_back(shape_[i]);
        st.push_back(strides_[i]);
    }
    matrix f = *this;
    f.set_layout(sh, st, type_, offset_);
    return f;
}

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

// ------------------------------------------------------------------------------------------
// Execution: execute passes recorded per binding
// ------------------------------------------------------------------------------------------
struct GraphCache {
    std::map<std::vector<const void*>, std::shared_ptr<void>> passes;
};

namespace {

constexpr size_t kMaxRecordedPasses = 8;
// Set while a pass is being recorded: a compiled function evaluated inside it launches its kernels
// directly, so they become part of the enclosing recording.
thread_local bool t_recording = false;

// Every device pointer a pass binds, in DFS order: each node's identity and output buffer (and a fused
// node's sibling outputs) and each leaf's data.  A recorded pass is valid exactly while these are unchanged.
void collect_bindings(matrix& m, std::vector<const void*>& sig, std::set<const Primitive*>& seen) {
    if (!m.has_tape()) {
        sig.push_back(m.data());
        return;
    }
    Primitive* p = m.tape_ptr().get();
    if (!seen.insert(p).second) return;
    sig.push_back(p);
    sig.push_back(p->out_buffer ? p->out_buffer->ptr : nullptr);
    p->extra_bindings(sig);
    for (matrix* in : p->inputs()) collect_bindings(*in, sig, seen);
}

void eval_roots(const std::vector<matrix*>& roots, EvalType t) {
    for (matrix* r : roots) {
        r->tape_ptr()->eval(*r, t);
        r->rebind_buffer(r->tape_ptr()->out_buffer);
    }
}

// One execute pass over compiled roots: replays the pass recorded for the current bindings, or records one
// (up to kMaxRecordedPasses per graph), or -- past that, or inside an enclosing recording -- launches the
// kernels directly.  A replay therefore never runs with another call's device pointers.
void run_pass(const std::vector<matrix*>& roots, GraphCache& cache, bool sync) {
    for (matrix* r : roots) r->tape_ptr()->clear_trace_checks();
    if (t_recording) {
        eval_roots(roots, EvalType::EXEC_TRACE);
        return;
    }
    std::vector<const void*> sig;
    std::set<const Primitive*> seen;
    for (matrix* r : roots) collect_bindings(*r, sig, seen);
    auto it = cache.passes.find(sig);
    if (it == cache.passes.end() && cache.passes.size() < kMaxRecordedPasses) {
        check(mtxc_graph_begin(), "mtxc_graph_begin");
        t_recording = true;
        t_defer_frees = true;
        try {
            eval_roots(roots, EvalType::EXEC_TRACE);
        } catch (...) {
            t_recording = false;
            t_defer_frees = false;
            void* g = nullptr;
            mtxc_graph_end(&g);
            if (g) mtxc_graph_destroy(g);
            release_deferred();
            throw;
        }
        t_recording = false;
        t_defer_frees = false;
        void* g = nullptr;
        const int rc_end = mtxc_graph_end(&g);
        release_deferred();
        check(rc_end, "mtxc_graph_end");
        it = cache.passes.emplace(sig, std::shared_ptr<void>(g, [](void* q) { mtxc_graph_destroy(q); })).first;
    }
    if (it != cache.passes.end()) check(mtxc_graph_launch(it->second.get()), "mtxc_graph_launch");
    else eval_roots(roots, EvalType::EXEC_TRACE);
    if (sync) check(mtxc_sync(), "mtxc_sync");
}

std::vector<matrix*> with_tapes(const std::vector<matrix*>& roots) {
    std::vector<matrix*> rs;
    for (matrix* r : roots)
        if (r && r->has_tape()) rs.push_back(r);
    return rs;
}

// ------------------------------------------------------------------------------------------
// Compiled functions (jit_graph_gpu / multi_jit_graph_gpu)
// ------------------------------------------------------------------------------------------
struct JitGraph {
    std::vector<std::shared_ptr<SwapLeafPrimitive>> leaves;
    std::vector<matrix> samples;  // the layouts callers' inputs must have
    std::vector<matrix> outputs;  // the compiled roots
    GraphCache cache;
};

// One call of a compiled function: its inputs and the nodes of its outputs.
struct JitCall {
    std::shared_ptr<JitGraph> g;
    std::vector<matrix> inputs;
    std::vector<std::weak_ptr<Primitive>> outs;
    std::vector<size_t> out_bytes;
    std::vector<std::shared_ptr<Buffer>> spare;  // for an output whose node no longer exists
    void prepare();                              // allocates every output buffer run() binds
    void run();
};

// The node a call's output carries (CompiledNodePrimitive / MultiInputCompilePrimitive): evaluating any
// output of the call runs the compiled graph once for all of them.
class JitOutputPrimitive : public Primitive {
public:
    JitOutputPrimitive(std::shared_ptr<JitCall> call, size_t index) : call_(std::move(call)), index_(index) {}
    void eval(matrix& out, EvalType t) override {
        for (matrix& in : call_->inputs) eval_input(in, t);
        allocate_output(*this, out);
        if (t == EvalType::COMPILE_TRACE) {
            call_->prepare();  // every output of the call has its buffer before any recorded pass
            return;
        }
        if (evaluated) return;
        call_->run();
    }
    void clear_trace_checks() override {
        evaluated = false;
        for (matrix& in : call_->inputs)
            if (in.has_tape()) in.tape_ptr()->clear_trace_checks();
    }
    std::vector<matrix*> inputs() override {
        std::vector<matrix*> v;
        for (matrix& in : call_->inputs) v.push_back(&in);
        return v;
    }
    const char* name() const override { return call_->outs.size() == 1 ? "CompiledNode" : "MultiInputCompile"; }
    void extra_bindings(std::vector<const void*>& sig) const override {
        for (size_t k = 0; k < call_->outs.size(); ++k)
            if (k != index_)
                if (auto n = call_->outs[k].lock()) sig.push_back(n->out_buffer ? n->out_buffer->ptr : nullptr);
    }

private:
    std::shared_ptr<JitCall> call_;
    size_t index_;
};

void JitCall::prepare() {
    if (spare.size() < outs.size()) spare.resize(outs.size());
    for (size_t k = 0; k < outs.size(); ++k) {
        auto n = outs[k].lock();
        if (n && !n->out_buffer) n->out_buffer = std::make_shared<Buffer>(out_bytes[k]);
        if (!n && !spare[k]) spare[k] = std::make_shared<Buffer>(out_bytes[k]);
    }
}

void JitCall::run() {
    // the caller's inputs go to the compiled graph's inputs (primitives.cpp:3938, 4187-4189) ...
    for (size_t i = 0; i < inputs.size(); ++i) {
        const matrix& in = inputs[i];
        const size_t bytes = std::max<uint64_t>(span(in.shape(), in.strides()), 1) * dtype_size(in.type());
        g->leaves[i]->out_buffer = std::make_shared<Buffer>(in.data(), bytes, in.buffer());
    }
    // ... and each owning node of the graph writes straight into the call's output (:3951-3956, 4191-4205)
    prepare();
    std::vector<std::shared_ptr<Primitive>> nodes(outs.size());
    for (size_t k = 0; k < outs.size(); ++k) {
        nodes[k] = outs[k].lock();
        g->outputs[k].tape_ptr()->out_buffer = nodes[k] ? nodes[k]->out_buffer : spare[k];
    }
    std::vector<matrix*> roots;
    for (matrix& o : g->outputs) roots.push_back(&o);
    run_pass(roots, g->cache, false);
    for (auto& n : nodes)
        if (n) n->evaluated = true;
    for (auto& leaf : g->leaves) leaf->out_buffer.reset();  // hold no caller memory between calls
}

}  // namespace

void matrix::eval() {
    Range range("mtx::eval");
    if (!tape_) return;
    if (tape_->evaluated) {
        rebind_buffer(tape_->out_buffer);
        return;
    }
    tape_->eval(*this, EvalType::EVAL_INSTANTLY);
    rebind_buffer(tape_->out_buffer);
    check(mtxc_sync(), "mtxc_sync");
}

void matrix::compile(const std::vector<matrix*>& roots) {
    Range range("mtx::compile");
    const std::vector<matrix*> rs = with_tapes(roots);
    if (rs.empty()) return;
    fuse_graph(rs);
    eval_roots(rs, EvalType::COMPILE_TRACE);
    auto cache = std::make_shared<GraphCache>();
    for (matrix* r : rs) r->graphs_ = cache;
}

void matrix::execute(const std::vector<matrix*>& roots) {
    Range range("mtx::execute");
    const std::vector<matrix*> rs = with_tapes(roots);
    if (rs.empty()) return;
    bool compiled = true;
    for (matrix* r : rs) compiled = compiled && r->tape_->out_buffer && r->graphs_;
    if (!compiled) compile(rs);
    run_pass(rs, *rs[0]->graphs_, true);
}

void matrix::compile() { compile(std::vector<matrix*>{this}); }
void matrix::execute() { execute(std::vector<matrix*>{this}); }

std::function<std::vector<matrix>(const std::vector<matrix>&)> matrix::multi_jit_graph_gpu(
    std::function<std::vector<matrix>(std::vector<matrix>)> func, const std::vector<matrix>& sample_inputs) {
    auto g = std::make_shared<JitGraph>();
    std::vector<matrix> inner;
    for (const matrix& s0 : sample_inputs) {
        matrix s = s0;
        if (s.tape_) s.eval();
        auto leaf = std::make_shared<SwapLeafPrimitive>();
        leaf->out_buffer = std::make_shared<Buffer>(
            s.data(), std::max<uint64_t>(span(s.shape_, s.strides_), 1) * dtype_size(s.type_), s.buffer_);
        matrix sl;
        sl.set_layout(s.shape_, s.strides_, s.type_);
        sl.set_tape(leaf);
        g->leaves.push_back(leaf);
        g->samples.push_back(sl);
        inner.push_back(sl);
    }
    g->outputs = func(inner);
    std::set<const Primitive*> distinct;
    for (const matrix& o : g->outputs) {
        // the reference refuses a graph whose output is its input (primitives.cpp:3953-3956)
        if (!o.tape_ || dynamic_cast<const SwapLeafPrimitive*>(o.tape_.get()))
            throw std::runtime_error("CompiledNodePrimitive: Head Tail Collision - cannot chop");
        if (!distinct.insert(o.tape_.get()).second)
            throw std::invalid_argument("multi_jit_graph_gpu: the outputs must be distinct nodes");
    }
    std::vector<matrix*> roots;
    for (matrix& o : g->outputs) roots.push_back(&o);
    compile(roots);
    for (auto& leaf : g->leaves) leaf->out_buffer.reset();  // calls bind their own inputs
    return [g](const std::vector<matrix>& inputs) -> std::vector<matrix> {
        if (inputs.size() != g->samples.size())
            throw std::invalid_argument("compiled function: wrong number of inputs");
        for (size_t i = 0; i < inputs.size(); ++i) {
            const matrix& a = inputs[i];
            const matrix& b = g->samples[i];
            if (a.shape() != b.shape() || a.strides() != b.strides() || a.type() != b.type())
                throw std::invalid_argument("compiled function: an input's shape, strides or dtype differ from the sample's");
        }
        auto call = std::make_shared<JitCall>();
        call->g = g;
        call->inputs = inputs;
        std::vector<matrix> outs;
        for (size_t k = 0; k < g->outputs.size(); ++k) {
            const matrix& o = g->outputs[k];
            matrix r;
            r.set_layout(o.shape(), o.strides(), o.type());
            auto node = std::make_shared<JitOutputPrimitive>(call, k);
            r.set_tape(node);
            call->outs.push_back(node);
            call->out_bytes.push_back(output_bytes(r));
            outs.push_back(r);
        }
        return outs;
    };
}

std::function<matrix(const matrix&)> matrix::jit_graph_gpu(std::function<matrix(matrix)> func, matrix sample) {
    auto multi = multi_jit_graph_gpu([func](std::vector<matrix> in) { return std::vector<matrix>{func(in[0])}; },
                                     {sample});
    return [multi](const matrix& input) -> matrix { return multi({input})[0]; };
}

void matrix::clear_trace_checks() {
    if (tape_) tape_->clear_trace_checks();
}

std::vector<uint8_t> matrix::to_host_bytes() const {
    matrix m = *this;
    if (m.tape_ && !m.tape_->evaluated && !m.graphs_) m.eval();
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

// ------------------------------------------------------------------------------------------
// Several GPUs (mtxc_comm_*)
// ------------------------------------------------------------------------------------------
std::string Communicator::unique_id() {
    std::string id(MTXC_COMM_ID_BYTES, '\0');
    check(mtxc_comm_unique_id(id.data(), id.size()), "mtxc_comm_unique_id");
    return id;
}

Communicator::Communicator(int nranks, int rank, const std::string& id, size_t buffer_bytes)
    : nranks_(nranks), rank_(rank) {
    if (nranks > 1 && id.size() != MTXC_COMM_ID_BYTES)
        throw std::invalid_argument("Communicator: the id must be MTXC_COMM_ID_BYTES bytes (Communicator::unique_id)");
    check(mtxc_comm_init(nranks, rank, nranks > 1 ? id.data() : nullptr, buffer_bytes), "mtxc_comm_init");
    if (int rc = mtxc_alloc(sizeof(int32_t), &token_)) {
        mtxc_comm_destroy();
        raise(rc, "mtxc_alloc");
    }
}

Communicator::~Communicator() {
    mtxc_sync();
    mtxc_comm_destroy();
    if (token_) mtxc_free(token_);
}

bool Communicator::peer_exchange() const {
    int peer = 0;
    check(mtxc_comm_status(&peer, nullptr), "mtxc_comm_status");
    return peer != 0;
}

bool Communicator::timed_out() {
    int late = 0;
    check(mtxc_comm_status(nullptr, &late), "mtxc_comm_status");
    return late != 0;
}

void Communicator::barrier() {
    // a rank's exchange starts after its earlier ones have finished (one stream) and completes only when
    // every rank's part of it has arrived, so when it completes here every rank is done writing into this
    // rank's buffers for the earlier ones
    check(mtxc_allreduce(MTXC_REDUCE_SUM, MTXC_INT32, token_, 1), "mtxc_allreduce");
    check(mtxc_sync(), "mtxc_sync");
}

matrix reduce_sharded(ReduceOp op, const matrix& local, const std::vector<int64_t>& first_rows, bool keepdims) {
    if (local.dims() == 0) throw std::invalid_argument("reduce_sharded: a 0-d matrix has no axis 0");
    const int code = (int)op;
    if (code < MTXC_REDUCE_SUM || code > MTXC_REDUCE_ARGMIN) throw std::invalid_argument("reduce_sharded: unknown op");
    const bool arg = op == ReduceOp::ArgMax || op == ReduceOp::ArgMin;
    int nranks = 0, rank = 0;
    check(mtxc_comm_size(&nranks, &rank), "reduce_sharded (needs a Communicator on this thread)");
    if (arg && first_rows.size() != (size_t)nranks)
        throw std::invalid_argument("reduce_sharded: ArgMax / ArgMin need first_rows for every rank");
    std::vector<size_m> out_shape = local.shape();
    if (keepdims) out_shape[0] = 1;
    else out_shape.erase(out_shape.begin());
    matrix out;
    out.set_layout(out_shape, row_major(out_shape), arg ? dtype::Int32 : local.type());
    out.set_tape(std::make_shared<ShardedReducePrimitive>(code, local, keepdims, out_shape, first_rows));
    return out;
}

}  // namespace mtx
