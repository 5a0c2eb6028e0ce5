// astype / copy for sm_100a: element type conversion over collapsed metadata.
//
// Replaces copyGPUinplace / copyGPUinplaceTypeCasted (Matrix.mm:1699-1922: the blit path for two
// contiguous operands and the Copy / TypeCasting kernels) behind matrix::astype(output, type, ...)
// (Matrix.mm:8400-8412), which the reference inserts in front of every mixed-dtype binary op
// (Matrix.mm:8313-8315).  The metadata is collapse_dims(in.shape, out.strides, in.strides) as in the
// CPU branch (matrix.h:1474-1544), whose element conversion is dtype_cast (matrix.h:260-267): a
// static_cast, through float between the two half types.
//
// Conversion rules (C++ static_cast on the reference's host compiler):
//   integer -> integer: the value modulo 2^bits;            integer -> float-like: round to nearest even;
//   float-like -> float-like: round to nearest even;         anything -> bool: x != 0 (NaN is true);
//   bool -> anything: 0 or 1;
//   float-like -> integer: truncation toward zero.  Defined by C++ only when the truncated value fits
//   the destination; outside that range the reference's result depends on its compiler, and this
//   kernel gives the low bits of the 64-bit truncation (saturated at the int64 range, NaN -> 0).
#include "elementwise.cuh"
#include "ops.cuh"

namespace mtxc {
namespace {

template <typename D, typename S>
struct CastOp {
    using Out = D;
    using In0 = S;
    using In1 = S;
    using In2 = S;
    static constexpr int kArity = 1;
    __device__ __forceinline__ D operator()(S x, S, S) const { return convert<D, S>(x); }
};

template <typename D>
int dispatch_src(int src_dtype, const ew::MapDesc& m, int sms, cudaStream_t stream, bool& known) {
    int rc = MTXC_OK;
    known = dispatch_dtype(src_dtype, [&](auto* stag) {
        using S = std::remove_pointer_t<decltype(stag)>;
        rc = ew::launch_map<CastOp<D, S>>(m, sms, stream);
    });
    return rc;
}

}  // namespace
}  // namespace mtxc

using namespace mtxc;

extern "C" int mtxc_astype(int dst_dtype, int src_dtype, void* dst, const void* src, uint32_t cdims,
                           const uint32_t* shape, const uint32_t* dst_strides, const uint32_t* src_strides) {
    if (int rc = require_init()) return rc;
    if (cdims > MTXC_MAX_DIMS) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_astype: cdims > MTXC_MAX_DIMS");
    if (cdims && (!shape || !dst_strides || !src_strides))
        return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_astype: null metadata pointer");
    auto known = [](int code) { return dispatch_dtype(code, [](auto*) {}); };
    if (!known(dst_dtype) || !known(src_dtype))
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_astype: no kernel for ") + dtype_name(src_dtype) +
                                                    " -> " + dtype_name(dst_dtype));
    if (cdims && product(shape, cdims) == 0) return MTXC_OK;  // nothing to convert
    if (!dst || !src) return fail(MTXC_ERR_INVALID_ARGUMENT, "mtxc_astype: null buffer");
    ThreadCtx& c = ctx();
    ew::MapDesc m{};
    m.dst = dst;
    m.src[0] = src;
    m.cdims = cdims;
    m.shape = shape;
    m.sd = dst_strides;
    m.ss[0] = src_strides;
    bool src_known = false;
    int rc = MTXC_OK;
    const bool dst_known = dispatch_dtype(dst_dtype, [&](auto* dtag) {
        using D = std::remove_pointer_t<decltype(dtag)>;
        rc = dispatch_src<D>(src_dtype, m, c.sm_count, c.stream(), src_known);
    });
    if (!dst_known || !src_known)
        return fail(MTXC_ERR_UNSUPPORTED_DTYPE, std::string("mtxc_astype: no kernel for ") + dtype_name(src_dtype) +
                                                    " -> " + dtype_name(dst_dtype));
    return rc;
}
