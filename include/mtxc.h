/*
 * mtxc.h -- C ABI of the B200 (sm_100a) backend for the reduce / broadcast hot path of
 * AlanAditya/matrix.
 *
 * The reference evaluates its axis reductions (Sum, Max, Min, ArgMax, ArgMin) and its
 * broadcasted binary ops (Add, Sub, Mul, Divide, Max, Min) either with CPU loops or by
 * encoding Metal compute kernels through one global GPUManager.  This library replaces the
 * Metal branch: every entry point below is what the reference's Phase-3 backend methods
 * would call in place of their `ExecutionDevice::METAL` branch.  Shapes and strides are the
 * reference's collapsed metadata (uint32 `size_m`, at most MTXC_MAX_DIMS axes), element
 * offsets are in elements, and a view offset is folded into the pointer, as the reference's
 * setBufferOrBytes does with its buffer offset.
 *
 * Conventions
 *   - Every function returns an int status (MTXC_OK == 0) unless stated otherwise; on
 *     failure mtxc_last_error() returns a message for the calling thread.
 *   - Kernels are enqueued on the calling thread's stream (mtxc_set_stream, else a stream
 *     the runtime creates in mtxc_init) and run asynchronously; mtxc_sync() waits.  Device
 *     faults surface at the next synchronising call.  This mirrors the reference's
 *     thread-local command buffer / encoder and its commit + waitUntilCompleted.
 *   - Inputs and outputs are caller-owned device buffers.  The hot-path calls never
 *     allocate or free: reductions that split an axis across CTAs use the calling thread's
 *     workspace, allocated in mtxc_init or supplied with mtxc_set_workspace.
 */
#ifndef MTXC_H
#define MTXC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MTXC_ABI_VERSION 1
#define MTXC_MAX_DIMS 8 /* MAX_TENSOR_DIMS, Mods/Utils.h:127 */

/* Status codes.  The reference throws std::runtime_error for a missing kernel / dtype
 * (Mods/GPUManager.h:62-71) and std::invalid_argument for shape errors (Matrix.mm:220);
 * a C++ caller rethrows these codes as the same exception types. */
enum {
    MTXC_OK = 0,
    MTXC_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad op code, cdims > MTXC_MAX_DIMS, ... */
    MTXC_ERR_UNSUPPORTED_DTYPE = 2,
    MTXC_ERR_SHAPE = 3,           /* incompatible broadcast shapes */
    MTXC_ERR_CUDA = 4,            /* a CUDA runtime call or kernel launch failed */
    MTXC_ERR_TIMEOUT = 5,         /* a bounded device-side wait gave up */
    MTXC_ERR_NOT_INITIALIZED = 6, /* mtxc_init was not called on this thread */
    MTXC_ERR_WORKSPACE = 7,       /* the thread's workspace cannot hold the split partials */
    MTXC_ERR_COMM = 8             /* NCCL missing or an NCCL call failed (multi-GPU entry points) */
};

/* dtype codes: identical to the reference's `enum class dtype` (matrix.h:35-51). */
enum {
    MTXC_FLOAT = 0,
    MTXC_FLOAT16 = 1,
    MTXC_UINT8 = 2,
    MTXC_INT32 = 3,
    MTXC_INT16 = 4,
    MTXC_UINT32 = 5,
    MTXC_UINT16 = 6,
    MTXC_BOOL = 7,
    MTXC_INT8 = 8,
    MTXC_COMPLEX64 = 9,
    MTXC_BFLOAT16 = 10,
    MTXC_INT64 = 11,
    MTXC_UINT64 = 12
};

/* Reduction ops: SumPrimitive, MaxReductionPrimitive, MinReductionPrimitive, ArgMaxPrimitive,
 * ArgMinPrimitive (primitives.cpp:2825-2971, 1967-2252, 7584-7799). */
enum { MTXC_REDUCE_SUM = 0, MTXC_REDUCE_MAX = 1, MTXC_REDUCE_MIN = 2, MTXC_REDUCE_ARGMAX = 3, MTXC_REDUCE_ARGMIN = 4 };

/* Broadcast binary ops: Addition/Subtraction/Multiplication/DivisionPrimitive,
 * Max/MinPrimitive (primitives.cpp:397-1046, 2515-2823) and EqualPrimitive (matrix::equal). */
enum { MTXC_BINARY_ADD = 0, MTXC_BINARY_SUB = 1, MTXC_BINARY_MUL = 2, MTXC_BINARY_DIV = 3, MTXC_BINARY_MAX = 4, MTXC_BINARY_MIN = 5,
       MTXC_BINARY_EQUAL = 6 };

/* Unary ops: ExpPrimitive (primitives.cpp:5332-5463), SqrtPrimitive. */
enum { MTXC_UNARY_EXP = 0, MTXC_UNARY_SQRT = 1 };

/* The make_pointwise family (Matrix.mm:13511-13604): GreaterPrimitive, LessPrimitive,
 * LogicalAndPrimitive, WherePrimitive, FloorPrimitive, FullPrimitive, Arctan2Primitive, ArcsinPrimitive. */
enum { MTXC_PW_GREATER = 0, MTXC_PW_LESS = 1, MTXC_PW_LOGICAL_AND = 2, MTXC_PW_WHERE = 3, MTXC_PW_FLOOR = 4, MTXC_PW_FULL = 5,
       MTXC_PW_ARCTAN2 = 6, MTXC_PW_ARCSIN = 7 };

/* ------------------------------------------------------------------------------------------
 * Runtime.  Replaces GPUManager's device / queue / per-thread command buffer layer
 * (Mods/GPUManager.h:47-600) and the no-copy buffer wrap buildMetalBuffer (matrix.h:677-680).
 * ---------------------------------------------------------------------------------------- */

/* Returns MTXC_ABI_VERSION. */
int mtxc_abi_version(void);

/* Binds the calling thread to CUDA device `device`, creates its stream and allocates its
 * workspace (MTXC_WORKSPACE_MB in the environment, default 64 MiB).  Replaces the
 * GPUManager constructor (Mods/GPUManager.h:53-54) and its lazy init* calls. */
int mtxc_init(int device);

/* Releases the calling thread's stream (if the runtime created it) and workspace (if the
 * runtime allocated it). */
int mtxc_shutdown(void);

/* Message describing the calling thread's last failure ("" when none).  The pointer stays
 * valid until the thread's next mtxc_* call. */
const char* mtxc_last_error(void);

int mtxc_device_count(int* count);

/* Makes `stream` (a cudaStream_t) the calling thread's stream.  NULL is CUDA's legacy default
 * stream, as everywhere in CUDA.  The caller keeps ownership. */
int mtxc_set_stream(void* stream);
/* Goes back to the stream the runtime created in mtxc_init. */
int mtxc_use_own_stream(void);
void* mtxc_get_stream(void);

/* Waits for all work on the calling thread's stream (the reference's commitCommandBuffer,
 * which commits and waits: Mods/GPUManager.h:558-562).  Reports asynchronous faults. */
int mtxc_sync(void);

/* Uses caller-owned device memory as the calling thread's workspace (replacing and freeing
 * one the runtime allocated).  bytes must be a multiple of 256 and ptr 256-byte aligned. */
int mtxc_set_workspace(void* ptr, size_t bytes);
/* Current workspace size in bytes of the calling thread. */
int mtxc_workspace_size(size_t* bytes);
/* Bytes of workspace mtxc_reduce would use for these arguments (0 when it needs none). */
int mtxc_reduce_workspace_bytes(int op, int dtype, uint32_t reduce_stride, uint32_t reduce_len, uint32_t cdims,
                                const uint32_t* shape, const uint32_t* dst_strides, const uint32_t* src_strides,
                                size_t* bytes);

/* Device memory (on the calling thread's device) and page-locked host memory. */
int mtxc_alloc(size_t bytes, void** dptr);
int mtxc_free(void* dptr);
int mtxc_host_alloc(size_t bytes, void** hptr);
int mtxc_host_free(void* hptr);
/* Asynchronous copies on the calling thread's stream. */
int mtxc_upload(void* dst_device, const void* src_host, size_t bytes);
int mtxc_download(void* dst_host, const void* src_device, size_t bytes);
int mtxc_copy_device(void* dst_device, const void* src_device, size_t bytes);
int mtxc_memset(void* dptr, int value, size_t bytes);

/* ------------------------------------------------------------------------------------------
 * Shape folding (host, no device work).  Same results as the reference's helpers, bit for
 * bit, including uint32 arithmetic.  Outputs are arrays of MTXC_MAX_DIMS entries; the
 * return value is the collapsed rank (`out_dims`).
 * ---------------------------------------------------------------------------------------- */

/* collapse_dims, 1 / 2 / 3 operands (Mods/Utils.mm:114-136, 138-166, 169-202). */
uint32_t mtxc_collapse_dims1(const uint32_t* shape, const uint32_t* s0, uint32_t dims, uint64_t size_cap,
                             uint32_t* out_shape, uint32_t* out_s0);
uint32_t mtxc_collapse_dims2(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, uint32_t dims,
                             uint64_t size_cap, uint32_t* out_shape, uint32_t* out_s0, uint32_t* out_s1);
uint32_t mtxc_collapse_dims3(const uint32_t* shape, const uint32_t* s0, const uint32_t* s1, const uint32_t* s2,
                             uint32_t dims, uint64_t size_cap, uint32_t* out_shape, uint32_t* out_s0,
                             uint32_t* out_s1, uint32_t* out_s2);
/* collapse_dims_reduce, 1 / 2 / 3 operands (Mods/Utils.mm:270-319, 321-376, 378-435). */
uint32_t mtxc_collapse_dims_reduce1(const uint32_t* shape, const uint32_t* s_out, uint32_t dims, int axis,
                                    int keep_dims, uint64_t size_cap, uint32_t* out_shape, uint32_t* out_s_out);
uint32_t mtxc_collapse_dims_reduce2(const uint32_t* shape, const uint32_t* s_out, const uint32_t* s_in,
                                    uint32_t dims, int axis, int keep_dims, int outer_collapsed,
                                    uint64_t size_cap, uint32_t* out_shape, uint32_t* out_s_out,
                                    uint32_t* out_s_in);
uint32_t mtxc_collapse_dims_reduce3(const uint32_t* shape, const uint32_t* s_out, const uint32_t* s_b,
                                    const uint32_t* s_c, uint32_t dims, int axis, int keep_dims,
                                    uint64_t size_cap, uint32_t* out_shape, uint32_t* out_s_out,
                                    uint32_t* out_s_b, uint32_t* out_s_c);

/* broadcast_shapes (Matrix.mm:161-232): right-aligned broadcast of (shape1, strides1, dim1)
 * against (shape2, strides2, dim2).  Fills the output shape and row-major strides and each
 * operand's broadcast shape and strides (0 on broadcast axes), max(dim1, dim2) entries
 * each.  Returns MTXC_ERR_SHAPE where the reference throws std::invalid_argument. */
int mtxc_broadcast_shapes(const uint32_t* shape1, const uint32_t* strides1, int dim1, const uint32_t* shape2,
                          const uint32_t* strides2, int dim2, uint32_t* out_shape, uint32_t* out_strides,
                          uint32_t* a_shape, uint32_t* a_strides, uint32_t* b_shape, uint32_t* b_strides);

/* promote_types (Matrix.mm:107-109, table matrix.h:166-180).  Returns the dtype code, or -1
 * for an out-of-range code. */
int mtxc_promote_types(int a, int b);

/* The make_pointwise collapse (Matrix.mm:13537-13555): axes of extent 1 are dropped, and an axis is
 * merged into the previous kept one when every input is contiguous across the two (stride of the
 * previous = stride * extent; stride-0 broadcasts merge) and the merged extent stays <= INT32_MAX.
 * out_shape: the output shape (out_dims entries).  in_strides: n_inputs rows of out_dims strides,
 * right-aligned to the output rank with 0 on broadcast axes (what make_pointwise builds as
 * all_strides).  Writes the collapsed shape (MTXC_MAX_DIMS entries) and n_inputs rows of
 * MTXC_MAX_DIMS collapsed strides (row i at out_strides + i * MTXC_MAX_DIMS); returns the collapsed
 * rank (0 for an empty output, as the reference skips the collapse when the count is 0, and for a
 * single element), or UINT32_MAX where the reference throws (out_dims > MTXC_MAX_DIMS, more than 2^32 - 1
 * output elements) and for n_inputs > 3 or null pointers. */
uint32_t mtxc_pointwise_collapse(const uint32_t* out_shape, uint32_t out_dims, const uint32_t* in_strides,
                                 uint32_t n_inputs, uint32_t* out_cshape, uint32_t* out_strides);

/* ------------------------------------------------------------------------------------------
 * Hot path.
 * ---------------------------------------------------------------------------------------- */

/* Axis reduction.  Replaces the METAL branch of matrix::sum / max / min / argmax / argmin
 * (Matrix.mm:15134-15186, 14841-14893, 14985-15037, 16211-16276, 16366-16431) and carries
 * exactly what those branches bind: the reduced axis' input stride and length, and the
 * primitive's collapsed metadata (collapse_dims_reduce with the output strides first).
 *
 * Output element gid (0 <= gid < prod(shape[0..cdims))) is written at dst[gid]; its input
 * run starts at src + sum_i (rem / dst_strides[i]) * src_strides[i] (rem %= dst_strides[i])
 * and holds reduce_len elements reduce_stride apart.  cdims == 0 means a single output.
 *
 * Results equal the reference CPU eval (Matrix.mm:15187-15207, 14894-14914, 15038-15058,
 * 16279-16302, 16434-16457): integer sums wrap like the reference's T accumulator; Max / Min
 * return the first element (lowest index) among the equal extremes, starting from
 * dtype_lowest / dtype_max, and never select NaN; ArgMax / ArgMin write int32 indices, the
 * first one on ties, 0 when no element beats the initial value.  Float sums are summed in a
 * different order (tree instead of sequential), so they agree within rounding.
 * dtypes: every reference dtype except Complex64 (MTXC_ERR_UNSUPPORTED_DTYPE): float, float16,
 * bfloat16, bool and the eight integer types.  Float16 / BFloat16 sums accumulate in fp32 and round
 * once, where the reference rounds every partial sum to the half type; Bool sums are a logical or
 * (C++ bool arithmetic). */
int mtxc_reduce(int op, int dtype, void* dst, const void* src, uint32_t reduce_stride, uint32_t reduce_len,
                uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides, const uint32_t* src_strides);

/* Fused statistics over one axis: matrix::mean / rms / norm (Matrix.mm:15220-15276), which the
 * reference composes from its primitives:
 *     MEAN  sum(x) / (float)n            RMS  sqrt(mean(x * x))            NORM  sqrt(sum(x * x))
 * with n = reduce_len.  One read of x instead of the three to five kernels of the composition; the
 * metadata is mtxc_reduce's.  The result is what the composition computes: x * x in the input dtype
 * (wrapping for integers), the sum rounded to the input dtype (integer sums wrap), one division by
 * (float)n converted to scalar_operand_type's dtype (matrix.h:1815-1846), one correctly rounded sqrt
 * in promote_types(type, Float16).  The output dtype therefore depends on the input dtype (and for
 * Float16 on n): mtxc_reduce_stat_dtype gives it.  Integer and Bool inputs give bit-exact results; float
 * sums are summed in a different order (fp32 tree instead of the reference's sequential sum in T), so
 * float results agree within rounding.  Workspace: as mtxc_reduce's SUM. */
enum { MTXC_STAT_MEAN = 0, MTXC_STAT_RMS = 1, MTXC_STAT_NORM = 2 };
int mtxc_reduce_stat(int stat, int dtype, void* dst, const void* src, uint32_t reduce_stride, uint32_t reduce_len,
                     uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides, const uint32_t* src_strides);
/* The dtype code mtxc_reduce_stat writes for (stat, input dtype, reduce_len), or -1:
 *   MEAN: Float -> Float, BFloat16 -> BFloat16, Float16 -> Float16 when n <= 65504 else Float, others -> Float
 *   RMS:  Float16 -> Float16 when n <= 65504 else Float, every other dtype -> Float
 *   NORM: Float16 and Bool -> Float16, every other dtype -> Float */
int mtxc_reduce_stat_dtype(int stat, int dtype, uint32_t reduce_len);

/* Max and ArgMax (op MAX or ARGMAX) or Min and ArgMin (op MIN or ARGMIN) from a single read of the
 * input: dst_values receives exactly what mtxc_reduce(MAX / MIN) writes and dst_indices exactly what
 * mtxc_reduce(ARGMAX / ARGMIN) writes, for the same metadata.  Serves the reference's
 * `x.max(axis)` + `x.argmax(axis)` pair (config 3) with half the HBM traffic, and the per-shard
 * partials of a sharded ArgMax. */
int mtxc_reduce_pair(int op, int dtype, void* dst_values, int32_t* dst_indices, const void* src,
                     uint32_t reduce_stride, uint32_t reduce_len, uint32_t cdims, const uint32_t* shape,
                     const uint32_t* dst_strides, const uint32_t* src_strides);

/* Merges the partial results of `parts` shards of a reduced axis, in shard order (the cross-GPU step
 * when the sharded axis is the reduced one).  part_values holds parts x outputs results, part-major
 * (dtype `dtype`; for ARGMAX / ARGMIN the shards' extreme values, from mtxc_reduce_pair).  SUM adds
 * them in order; MAX / MIN keep the first shard's value unless a later one is strictly better;
 * ARGMAX / ARGMIN pick the shard the same way and write part_indices[p][j] + index_offsets[p]
 * (index_offsets: host array, the first element of each shard's slice) to dst_indices, and the value to
 * dst unless dst is NULL.  parts <= 256.  Results equal the unsharded reduction's (float sums within
 * rounding). */
int mtxc_merge_partials(int op, int dtype, void* dst, int32_t* dst_indices, const void* part_values,
                        const int32_t* part_indices, const int64_t* index_offsets, uint32_t parts,
                        uint64_t outputs);

/* mtxc_reduce for callers that cannot allocate device memory.  No counterpart in the reference.
 *
 * Some callers of this library may not call cudaMalloc: code that runs inside another framework's
 * memory manager (which owns every byte of device memory and forbids side allocations), latency-
 * critical loops that cannot afford the device-wide synchronisation cudaMalloc / cudaFree imply, or
 * deployments whose memory budget is fixed up front.  mtxc_reduce needs scratch memory when it splits a
 * reduced axis across CTAs (the per-split partials), and takes it from the thread's workspace, which
 * mtxc_init allocates.  This entry point computes the same reduction, with the same kernels and the same
 * arguments, but keeps the partials in a statically sized array that is part of the library's device
 * image (MTXC_NOALLOC_SCRATCH_BYTES, 4 MiB; every GPU that loads the library holds it until the process
 * exits).  It calls no allocator: no cudaMalloc, cudaFree or library routine that allocates.  (Call
 * mtxc_init with MTXC_WORKSPACE_MB=0 in the environment to keep the runtime from allocating its own
 * workspace as well.)
 *
 * Results: identical to mtxc_reduce's whenever mtxc_reduce's workspace holds the same split (the default
 * 64 MiB workspace always does).  With a smaller workspace mtxc_reduce splits the axis less, so a float
 * Sum may round differently -- both stay within the float-sum tolerance of the CPU -- while integer sums,
 * Max / Min and ArgMax / ArgMin are identical whatever the split.
 *
 *   - A reduction whose partials would need more than MTXC_NOALLOC_SCRATCH_BYTES is rejected with
 *     MTXC_ERR_WORKSPACE and a message giving both sizes; mtxc_reduce_workspace_bytes tells in advance.
 *   - The first call on each device looks up the array's device address with that device current
 *     (cudaGetSymbolAddress) and caches it; make that first call before any stream capture.  The cache
 *     assumes the device is not reset behind the library: after a cudaDeviceReset, call mtxc_shutdown
 *     (which drops the device's cached address) and mtxc_init before the next call.
 *   - All calls on a device share the one array, and it keeps whatever the last call left in it.
 *     Nothing in it has to start at zero (every partial is written before it is read), but calls that
 *     overlap on the GPU -- on different streams or from different threads -- race on it: order them. */
#define MTXC_NOALLOC_SCRATCH_BYTES (4u << 20)
int mtxc_reduce_noalloc(int op, int dtype, void* dst, const void* src, uint32_t reduce_stride,
                        uint32_t reduce_len, uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides,
                        const uint32_t* src_strides);

/* Broadcasted binary op.  Replaces add/subtract/multiply/divide_gpu_brodcasted
 * (Matrix.mm:7709-8239) and the METAL branch of matrix::max / min(other, result, dev)
 * (Matrix.mm:13396-13450, 14701-14755), binding the primitive's collapsed_dims_3:
 * shape, the result strides, and the per-operand strides (0 on broadcast axes).
 *
 * Result element gid (0 <= gid < prod(shape)) is written at r[gid] and equals
 * a[sum idx_i * a_strides[i]] op b[sum idx_i * b_strides[i]] with idx_i decoded from gid by
 * the result strides (Matrix.mm:7475-7498).  cdims == 0 is the scalar case.  Float results
 * are bit-exact with the reference CPU (one IEEE-rounded op per element, no contraction);
 * Max / Min keep `a` unless `b` is strictly greater / smaller (std::max / std::min).
 * Integer results wrap; integer division by zero is undefined, as in the reference.
 * Float16 / BFloat16 ops compute in fp32 and round once, which is the correctly rounded half result
 * (bit-exact with the reference CPU); Bool follows C++ bool arithmetic.
 * Both operands have dtype `dtype` (the reference promotes with astype first). */
int mtxc_broadcast_binary(int op, int dtype, void* r, const void* a, const void* b, uint32_t cdims,
                          const uint32_t* shape, const uint32_t* r_strides, const uint32_t* a_strides,
                          const uint32_t* b_strides);

/* a op b for operands of different dtypes with the promotion fused in: the result equals
 * mtxc_broadcast_binary(op, dtype, ...) applied to the operands after mtxc_astype to dtype =
 * promote_types(a_dtype, b_dtype), which is what the reference evaluates (astype of the operand whose dtype
 * differs, then the op: Matrix.mm:8312-8382), bit for bit -- but in one pass, without writing and
 * re-reading a converted copy.  Same metadata as mtxc_broadcast_binary (the strides of the operands as
 * given; the reference's astype keeps them).  Supported: op ADD, SUB, MUL, DIV or EQUAL; any two different
 * operand dtypes but Complex64, whether the promoted dtype is one of them (Float with Int32, Int64 with
 * Int32, ...) or a third (Float16 with Int32 -> Float, UInt8 with Int8 -> Int16, ...).  Complex64:
 * MTXC_ERR_UNSUPPORTED_DTYPE; dtype other than promote_types(a_dtype, b_dtype), or a_dtype == b_dtype:
 * MTXC_ERR_INVALID_ARGUMENT. */
int mtxc_broadcast_binary_mixed(int op, int dtype, int a_dtype, int b_dtype, void* r, const void* a, const void* b,
                                uint32_t cdims, const uint32_t* shape, const uint32_t* r_strides,
                                const uint32_t* a_strides, const uint32_t* b_strides);

/* Elementwise unary op over collapse_dims(shape, out strides, in strides) metadata
 * (Matrix.mm:6798-6925, 6934-7065), on Float or Float16 (the frontends promote other dtypes first).
 * EXP: CUDA expf, within 2 ulp of the CPU's std::exp (Float16: that result rounded once).  SQRT: the
 * correctly rounded square root, bit-exact with std::sqrt. */
int mtxc_unary(int op, int dtype, void* dst, const void* src, uint32_t cdims, const uint32_t* shape,
               const uint32_t* dst_strides, const uint32_t* src_strides);

/* Element type conversion and strided copy: matrix::astype(output, type, ...) (Matrix.mm:8400-8412)
 * through copyGPUinplace / copyGPUinplaceTypeCasted (Matrix.mm:1699-1922).  Metadata:
 * collapse_dims(in.shape, out.strides, in.strides, INT32_MAX), as the reference computes it
 * (matrix.h:1481).  Element gid's position is decoded from shape; dst[sum idx*dst_strides] =
 * dtype_cast<Dst>(src[sum idx*src_strides]) (matrix.h:260-267): integers wrap, conversions to a
 * float-like type round to nearest even (half <-> bfloat16 through float), conversions to Bool test
 * x != 0, float-likes truncate toward zero into integers (defined when the result fits; outside the
 * destination's range the low bits of the 64-bit truncation are written).  Every dtype pair except
 * Complex64; dst_dtype == src_dtype is a copy. */
int mtxc_astype(int dst_dtype, int src_dtype, void* dst, const void* src, uint32_t cdims, const uint32_t* shape,
                const uint32_t* dst_strides, const uint32_t* src_strides);

/* The make_pointwise family over mtxc_pointwise_collapse metadata.  The output is contiguous (element
 * gid at dst[gid]); input k's element is at inputs[k][sum idx_i * strides[k * MTXC_MAX_DIMS + i]] (the
 * layout of the reference's ElementwiseDims::strides[3][MAX_TENSOR_DIMS]).  cdims == 0 is one element
 * at offset 0.  dtype is the inputs' common dtype (the frontends cast first):
 *   GREATER, LESS (2 inputs of dtype)      -> Bool: a > b, a < b (greater/less_backend_cpu)
 *   LOGICAL_AND (2 Bool inputs)             -> Bool: a && b
 *   WHERE (Bool cond, a, b of dtype)        -> dtype: cond ? a : b (inputs ordered cond, a, b)
 *   FLOOR (1 input)                         -> dtype: floor for float-likes, identity otherwise
 *   FULL (1 input, the broadcast value)     -> dtype: the value
 *   ARCTAN2 (2 Float inputs)                -> Float: atan2(a, b) (arctan2_backend_cpu, Matrix.mm:13608)
 *   ARCSIN (1 Float input)                  -> Float: asin(x)     (arcsin_backend_cpu, Matrix.mm:13680)
 * Results are bit-exact with the CPU backends (Matrix.mm:13741-14166), except ARCTAN2 / ARCSIN, which call
 * CUDA's atan2f / asinf: within 3 ulp of the CPU's std::atan2 / std::asin (the frontends cast the inputs
 * to Float first, Matrix.mm:13573-13580).  The output must not exceed
 * 2^32 - 1 elements (make_pointwise's limit).  An empty output needs no call: its collapsed rank is 0,
 * as for a single element, and the reference's backends return before reading anything
 * (`if (!output.total_size) return;`). */
int mtxc_pointwise(int op, int dtype, void* dst, const void* const* inputs, uint32_t n_inputs, uint32_t cdims,
                   const uint32_t* shape, const uint32_t* strides);

/* matrix::arange(start, stop, step, type) (Matrix.mm:13595-13604) evaluated: dst[i] = start + i * step for
 * i < count (count = max(0, ceil((stop - start) / step)), computed by the frontend), replacing
 * arange_backend_gpu (Matrix.mm:14407).  start and step are device pointers to one element of dtype each
 * (the primitive's two scalar inputs, dtype_cast to the output type); dst is contiguous.  Integers:
 * (T)((uint64)start + (uint64)i * (uint64)step), wrapping; Float / Float16 / BFloat16:
 * float(start) + float(i) * float(step) with each operation rounded once (no fused multiply-add), then
 * rounded to the dtype.  Bit-exact with the CPU backend (Matrix.mm:14167-14180).  Bool:
 * MTXC_ERR_UNSUPPORTED_DTYPE, as arange refuses it; count > 2^32 - 1: MTXC_ERR_SHAPE. */
int mtxc_arange(int dtype, void* dst, const void* start, const void* step, uint64_t count);

/* Fused evaluation of the reference's softmax trace over the last axis of contiguous float rows
 *     m = x.max(-1, true); e = matrix::exp(x - m); y = e / e.sum(-1, true)
 * (MaxReduction, Subtraction, Exp, Sum and Division primitives; benchmark config 5a): x is read once
 * and y written once.  Element-wise the trace's arithmetic (same max, x - m, expf) except for the order
 * of the fp32 additions in the row sum and y = e * (1 / s), one correctly rounded reciprocal per row,
 * within 1 ulp of the trace's e / s.  Rows start row_stride elements apart;
 * row_len must be a multiple of 4, rows 16-byte aligned and row_len <= MTXC_SOFTMAX_MAX_ROW, else
 * MTXC_ERR_INVALID_ARGUMENT (evaluate the unfused trace instead).  A compiled trace substitutes it
 * for those five primitives when their shapes match (no counterpart kernel in the reference, which
 * runs the five primitives one by one). */
#define MTXC_SOFTMAX_MAX_ROW 65536u
int mtxc_softmax_lastdim(int dtype, void* dst, const void* src, uint64_t rows, uint32_t row_len,
                         uint64_t src_row_stride, uint64_t dst_row_stride);

/* ------------------------------------------------------------------------------------------
 * Multi-GPU: one communicator per GPU for reductions over an axis sharded across the GPUs of a node
 * (benchmark configs 4 and 5b).  The reference drives a single Metal device through one GPUManager
 * (Mods/GPUManager.h:53-54); these entry points are the multi-device half of the layer that replaces
 * it (the `mtxc_comm_init` / `mtxc_allreduce` exports a multi-GPU drop-in needs).  One process (or host
 * thread) per GPU; each calls mtxc_init(device) and then mtxc_comm_init with the same unique id.
 * NCCL (libnccl.so.2) is loaded at run time, reusing the copy already in the process if there is one;
 * a one-rank communicator does not need it.
 *
 * The exchange is an all-gather of the per-rank partials plus a merge in rank order on every rank: every
 * rank ends with the same result, float sums are deterministic, and Max / ArgMax keep the first-index rule
 * across GPUs.  When every rank drives its own GPU of one node it runs as one kernel over NVLink peer
 * memory (each rank stores its partials into every rank's buffer, raises a flag there and merges once
 * every rank's flag has arrived); otherwise as an NCCL all-gather and a merge kernel.  Everything is
 * enqueued on the calling thread's stream; like every collective, all ranks must make the same calls in
 * the same order, and one communicator's calls must not overlap on the GPU (issue them on one stream, or
 * order them with events).
 * ---------------------------------------------------------------------------------------- */
#define MTXC_COMM_ID_BYTES 128

/* Writes a new unique id (MTXC_COMM_ID_BYTES bytes) for one communicator.  Call on one rank and hand
 * the bytes to the others out of band (a store, MPI, a file).  MTXC_ERR_COMM when NCCL is missing. */
int mtxc_comm_unique_id(void* id, size_t bytes);

/* Joins the calling thread (bound to its device by mtxc_init) to a communicator of nranks ranks as
 * rank `rank`.  Blocks until all nranks ranks have joined (ncclCommInitRank), then sets up the peer
 * exchange (collectively; see mtxc_comm_status).  Allocates the buffers the exchanges use, each about
 * buffer_bytes (0: 16 MiB; at least 64 KiB with several ranks; the same value on every rank), once, here:
 * the exchanges never allocate.  One communicator per thread; mtxc_comm_destroy (or mtxc_shutdown) releases
 * it.  nranks == 1 needs no id and no NCCL. */
int mtxc_comm_init(int nranks, int rank, const void* id, size_t buffer_bytes);
/* Waits for the thread's stream and releases its communicator.  With the peer exchange, every rank's last
 * exchange must have finished before any rank destroys (synchronise every rank, then a barrier): a rank still
 * running one writes into the others' buffers. */
int mtxc_comm_destroy(void);
int mtxc_comm_size(int* nranks, int* rank);
/* *peer_exchange (if non-NULL): 1 when the exchanges run as one kernel over peer memory (every rank on its
 * own GPU of one node, the ranks' exchange buffers mapped into each other with CUDA IPC at mtxc_comm_init;
 * MTXC_COMM_PEER=0 in the environment keeps the NCCL all-gather + merge instead), else 0.  *timed_out (if
 * non-NULL): waits for the thread's stream, then reports whether an exchange since the last query gave up
 * waiting for a rank (a rank that never made the call: the peer exchange's waits are bounded -- 2^22 polls
 * of the rank's flag, each followed by a short sleep, or MTXC_COMM_SPIN_LIMIT polls -- so it returns instead
 * of hanging, and its outputs are not valid) and clears the flag. */
int mtxc_comm_status(int* peer_exchange, int* timed_out);

/* A reduction over an axis that is sharded across the ranks: this rank holds a contiguous slice of the
 * reduced axis, described exactly as for mtxc_reduce (reduce_len = the slice's length, which may be 0).
 * On return every rank's dst holds the reduction over the whole axis, as mtxc_reduce over the unsharded
 * tensor would give it: integer sums, Max / Min and ArgMax / ArgMin bit-exact; float sums add the ranks'
 * partial sums in rank order (within rounding of the unsharded sum).  ArgMax / ArgMin write int32 global
 * indices and need index_offsets: a host array of nranks entries, the global index of each rank's first
 * element (the same array on every rank); it is ignored (may be NULL) for the other ops.  Steps, on the
 * thread's stream: the local reduction into this rank's slot of the gather buffer, the in-place NCCL
 * all-gather, the ordered merge into dst.  MTXC_ERR_WORKSPACE when nranks x outputs partials do not fit
 * the communicator's buffer. */
int mtxc_reduce_sharded(int op, int dtype, void* dst, const void* src, uint32_t reduce_stride, uint32_t reduce_len,
                        uint32_t cdims, const uint32_t* shape, const uint32_t* dst_strides,
                        const uint32_t* src_strides, const int64_t* index_offsets);

/* In-place all-reduce of `count` elements of buf (op SUM, MAX or MIN) across the ranks: every rank ends
 * with buf = the ranks' buffers combined in rank order (SUM: ordered adds, integers wrap; MAX / MIN: a
 * later rank's value replaces an earlier one's only when strictly better).  Identical on every rank. */
int mtxc_allreduce(int op, int dtype, void* buf, uint64_t count);

/* ------------------------------------------------------------------------------------------
 * Compiled trace: record the kernels one execute pass enqueues and replay them.  The B200
 * form of the reference's compile-once / execute-many model (Matrix.mm:8452-8475).
 * ---------------------------------------------------------------------------------------- */

/* Starts capturing the calling thread's stream into a CUDA graph. */
int mtxc_graph_begin(void);
/* Ends the capture and instantiates it; *graph receives an opaque handle. */
int mtxc_graph_end(void** graph);
/* Replays a captured graph on the calling thread's stream. */
int mtxc_graph_launch(void* graph);
int mtxc_graph_destroy(void* graph);

#ifdef __cplusplus
}
#endif

#endif /* MTXC_H */
