// Mixed-dtype broadcast binary ops with the promotion fused in, for sm_100a.
//
// The reference evaluates `a + b` with a.type != b.type as astype of the operand(s) whose dtype is not
// promote_types(a.type, b.type), followed by the op (Matrix.mm:8312-8382, 14451-14466): a promoted copy
// of the operand is written and read back.  astype is element-wise and, in that path, keeps the
// operand's strides (astype(common) without make_contig, Matrix.mm:8384-8398), so converting each element
// as the op reads it gives the same bits with one pass over the data: for an int32 [N] + float [N] add,
// 12 bytes per element move instead of 20.
//
// Covered here: a Float result with one Float operand and one operand of any other dtype (the common
// mixed case: an integer, half or Bool tensor meeting a float one), for the promoting ops Add, Sub, Mul,
// Div and Equal.  The metadata is the op's own (broadcast_shapes + collapse_dims over the result and
// the two operands).  Other combinations use mtxc_astype then mtxc_broadcast_binary.
#include "elementwise.cuh"
#include "ops.cuh"

namespace mtxc {
namespace {

template <int OP, typename SA, typename SB>
struct MixedOp {
    using Out = float;
    using In0 = SA;
    using In1 = SB;
    using In2 = SA;
    static constexpr int kArity = 2;
    __device__ __forceinline__ float operator()(SA a, SB b, SA) const {
        return apply<OP, float>(convert<float, SA>(a), convert<float, SB>(b));
    }
};

template <int OP>
int launch_mixed(int a_dtype, int b_dtype, const ew::MapDesc& m, int sms, cudaStream_t st, bool& known) {
    int rc = MTXC_OK;
    if (a_dtype == MTXC_FLOAT) {
        known = dispatch_dtype(b_dtype, [&](auto* tag) {
            using SB = std::remove_pointer_t<decltype(tag)>;
            rc = ew::launch_map<MixedOp<OP, float, SB>>(m, sms, st);
        });
    } else {
        known = dispatch_dtype(a_dtype, [&](auto* tag) {
            using SA = std::remove_pointer_t<decltype(tag)>;
            rc = ew::launch_map<MixedOp<OP, SA, float>>(m, sms, st);
        });
    }
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
    if (dtype != MTXC_FLOAT || (a_dtype != MTXC_FLOAT && b_dtype != MTXC_FLOAT))
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, "mtxc_broadcast_binary_mixed: needs a Float result and a Float "
                                                "operand (use mtxc_astype + mtxc_broadcast_binary)");
    if (mtxc_promote_types(a_dtype, b_dtype) != dtype)
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_broadcast_binary_mixed: dtype is not promote_types(a, b)");
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
    switch (op) {
        case MTXC_BINARY_ADD: rc = launch_mixed<MTXC_BINARY_ADD>(a_dtype, b_dtype, m, c.sm_count, c.stream(), known); break;
        case MTXC_BINARY_SUB: rc = launch_mixed<MTXC_BINARY_SUB>(a_dtype, b_dtype, m, c.sm_count, c.stream(), known); break;
        case MTXC_BINARY_MUL: rc = launch_mixed<MTXC_BINARY_MUL>(a_dtype, b_dtype, m, c.sm_count, c.stream(), known); break;
        case MTXC_BINARY_DIV: rc = launch_mixed<MTXC_BINARY_DIV>(a_dtype, b_dtype, m, c.sm_count, c.stream(), known); break;
        default: rc = launch_mixed<MTXC_BINARY_EQUAL>(a_dtype, b_dtype, m, c.sm_count, c.stream(), known); break;
    }
    if (!known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_broadcast_binary_mixed: no kernel for ") +
                                                    dtype_name(a_dtype) + " with " + dtype_name(b_dtype));
    return rc;
}
