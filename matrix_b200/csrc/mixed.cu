// Mixed-dtype broadcast binary ops with the promotion fused in, for sm_100a.
//
// The reference evaluates `a + b` with a.type != b.type as astype of the operand(s) whose dtype is not
// promote_types(a.type, b.type), followed by the op (Matrix.mm:8312-8382, 14451-14466): a promoted copy
// of the operand is written and read back.  astype is element-wise and, in that path, keeps the
// operand's strides (astype(common) without make_contig, Matrix.mm:8384-8398), so converting each element
// as the op reads it gives the same bits with one pass over the data: for an int32 [N] + float [N] add,
// 12 bytes per element move instead of 20.
//
// Covered here: every pair of operand dtypes whose promoted dtype is one of the two (a Float result with a
// Float operand and any other; Int64 with Int32 or a narrower integer; a half type with Bool; ...), for the
// promoting ops Add, Sub, Mul, Div and Equal.  The operand of the result's dtype is read as it is, the other
// converted as it is read (convert<>, the conversion of mtxc_astype), and the op is apply<> in the result
// dtype, as in mtxc_broadcast_binary.  Pairs that promote to a third dtype (e.g. Float16 with Int32 ->
// Float) are in mixed3.cu, reached from the same entry point.  The metadata is the op's own (broadcast_shapes +
// collapse_dims over the result and the two operands).
#include "mixed.cuh"

namespace mtxc {
namespace {

// D: the result dtype, which one operand (`a` when d_is_a) already has; the other operand's dtype is
// `other`.  Instantiates the kernel only for pairs the promotion table maps to D.
template <int OP>
int launch_mixed(int dtype, int other, bool d_is_a, const ew::MapDesc& m, int sms, cudaStream_t st, bool& known) {
    int rc = MTXC_OK;
    bool has_kernel = false;
    dispatch_dtype(dtype, [&](auto* dtag) {
        using D = std::remove_pointer_t<decltype(dtag)>;
        dispatch_dtype(other, [&](auto* stag) {
            using S = std::remove_pointer_t<decltype(stag)>;
            if constexpr (!std::is_same_v<D, S> && promote_code(code_of<D>(), code_of<S>()) == code_of<D>()) {
                has_kernel = true;
                if (d_is_a) rc = ew::launch_map<MixedOp<OP, D, D, S>>(m, sms, st);
                else rc = ew::launch_map<MixedOp<OP, D, S, D>>(m, sms, st);
            }
        });
    });
    known = has_kernel;
    return rc;
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_broadcast_binary_mixed(int op, int dtype, int a_dtype, int b_dtype, void* r, const void* a,
                                           const void* b, uint32_t cdims, const uint32_t* shape,
                                           const uint32_t* r_strides, const uint32_t* a_strides,
                                           const uint32_t* b_strides) {
    if (int rc = require_init()) return rc;
    if (op != MTXC_BINARY_ADD && op != MTXC_BINARY_SUB && op != MTXC_BINARY_MUL && op != MTXC_BINARY_DIV &&
        op != MTXC_BINARY_EQUAL)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: only the promoting ops (add, sub, mul, "
                                               "div, equal)");
    if (mtxc_promote_types(a_dtype, b_dtype) != dtype)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: dtype is not promote_types(a, b)");
    if (a_dtype == b_dtype)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: operands of one dtype (use "
                                               "mtxc_broadcast_binary)");
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: cdims > MTXC_MAX_DIMS");
    if (cdims && (!shape || !r_strides || !a_strides || !b_strides))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: null metadata pointer");
    if (cdims && product(shape, cdims) == 0) return MTXC_OK;
    if (!r || !a || !b) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: null buffer");
    ew::MapDesc m{};
    m.dst = r;
    m.src[0] = a;
    m.src[1] = b;
    m.cdims = cdims;
    m.shape = shape;
    m.sd = r_strides;
    m.ss[0] = a_strides;
    m.ss[1] = b_strides;
    ThreadCtx& c = ctx();
    bool known = false;
    int rc = MTXC_OK;
    if (a_dtype != dtype && b_dtype != dtype) {  // promoted to a third dtype (mixed3.cu)
        rc = launch_mixed3(op, dtype, a_dtype, b_dtype, m, c.sm_count, c.stream(), known);
        if (!known)
            return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_broadcast_binary_mixed: no kernel for ") +
                                                        dtype_name(a_dtype) + " with " + dtype_name(b_dtype));
        return rc;
    }
    const bool d_is_a = a_dtype == dtype;
    const int other = d_is_a ? b_dtype : a_dtype;
    switch (op) {
        case MTXC_BINARY_ADD: rc = launch_mixed<MTXC_BINARY_ADD>(dtype, other, d_is_a, m, c.sm_count, c.stream(), known); break;
        case MTXC_BINARY_SUB: rc = launch_mixed<MTXC_BINARY_SUB>(dtype, other, d_is_a, m, c.sm_count, c.stream(), known); break;
        case MTXC_BINARY_MUL: rc = launch_mixed<MTXC_BINARY_MUL>(dtype, other, d_is_a, m, c.sm_count, c.stream(), known); break;
        case MTXC_BINARY_DIV: rc = launch_mixed<MTXC_BINARY_DIV>(dtype, other, d_is_a, m, c.sm_count, c.stream(), known); break;
        default: rc = launch_mixed<MTXC_BINARY_EQUAL>(dtype, other, d_is_a, m, c.sm_count, c.stream(), known); break;
    }
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_broadcast_binary_mixed: no kernel for ") +
                                                    dtype_name(a_dtype) + " with " + dtype_name(b_dtype));
    return rc;
}
