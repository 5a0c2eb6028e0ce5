// Mixed-dtype broadcast binary ops whose promoted dtype is neither operand's (Float16 with Int32 -> Float,
// UInt8 with Int8 -> Int16, Int16 with UInt32 -> Int32, ...; 26 of the 66 dtype pairs), for sm_100a.
//
// The reference converts both operands with astype(promote_types(a, b)) and then runs the op in that
// dtype (Matrix.mm:8312-8382): two converted copies are written and read back.  Here both operands are
// converted as the op reads them (convert<>, the conversion of mtxc_astype) and the op is apply<> in the
// result dtype, as mtxc_broadcast_binary computes it: the same bits in one pass.  Reached through
// mtxc_broadcast_binary_mixed; the pairs whose promoted dtype is one of the two live in mixed.cu.
#include "mixed.cuh"

namespace mtxc {
namespace {

template <int OP>
int launch_third(int dtype, int a_dtype, int b_dtype, const ew::MapDesc& m, int sms, cudaStream_t st, bool& known) {
    int rc = MTXC_OK;
    bool has_kernel = false;
    dispatch_dtype(dtype, [&](auto* dtag) {
        using D = std::remove_pointer_t<decltype(dtag)>;
        // only Float, Int16 and Int32 are the promoted dtype of a pair of two other dtypes
        if constexpr (std::is_same_v<D, float> || std::is_same_v<D, int16_t> || std::is_same_v<D, int32_t>) {
            dispatch_dtype(a_dtype, [&](auto* atag) {
                using SA = std::remove_pointer_t<decltype(atag)>;
                dispatch_dtype(b_dtype, [&](auto* btag) {
                    using SB = std::remove_pointer_t<decltype(btag)>;
                    constexpr int d = code_of<D>(), a = code_of<SA>(), b = code_of<SB>();
                    if constexpr (a != d && b != d && a != b && promote_code(a, b) == d) {
                        has_kernel = true;
                        rc = ew::launch_map<MixedOp<OP, D, SA, SB>>(m, sms, st);
                    }
                });
            });
        }
    });
    known = has_kernel;
    return rc;
}

}  // namespace

int launch_mixed3(int op, int dtype, int a_dtype, int b_dtype, const ew::MapDesc& m, int sms, cudaStream_t st,
                  bool& known) {
    switch (op) {
        case MTXC_BINARY_ADD: return launch_third<MTXC_BINARY_ADD>(dtype, a_dtype, b_dtype, m, sms, st, known);
        case MTXC_BINARY_SUB: return launch_third<MTXC_BINARY_SUB>(dtype, a_dtype, b_dtype, m, sms, st, known);
        case MTXC_BINARY_MUL: return launch_third<MTXC_BINARY_MUL>(dtype, a_dtype, b_dtype, m, sms, st, known);
        case MTXC_BINARY_DIV: return launch_third<MTXC_BINARY_DIV>(dtype, a_dtype, b_dtype, m, sms, st, known);
        default: return launch_third<MTXC_BINARY_EQUAL>(dtype, a_dtype, b_dtype, m, sms, st, known);
    }
}

}  // namespace mtxc
