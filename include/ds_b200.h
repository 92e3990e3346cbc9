/*
 * ds_b200.h -- C ABI of the B200 (sm_100a) double-single (DS) operator library
 * (libds_b200.so).
 *
 * A DS value is a pair of float32 (hi, lo) whose exact sum carries about 48
 * significant bits.  Packed DS tensors have a trailing dimension of 2 with hi
 * at even and lo at odd offsets; SoA DS tensors are two f32 tensors of the
 * same shape.
 *
 * Each entry point replaces one XLA-FFI custom-call target of the reference
 * (rcast915/ds-experiment) and keeps its operands, attribute, result and
 * shape checks; the citation above each declaration names the handler it
 * replaces.  Differences from the reference, all deliberate:
 *   - every op runs as sm_100a CUDA on the caller's stream (the reference's
 *     CPU handlers loop on the host; its three CUDA handlers launch on the
 *     legacy default stream and call cudaDeviceSynchronize).  No entry point
 *     synchronises; results are ready when the stream reaches them.
 *   - buffers are described by ds_buffer (device pointer + dims), which is
 *     what an XLA-FFI adapter gets from ffi::Buffer::untyped_data() and
 *     dimensions(); no XLA or torch type appears here.
 *   - ds_reduce and ds_dot_general are new targets for the DS pass's reduce
 *     and dot_general rewrites; they take caller-provided workspace (XLA's
 *     scratch allocator in an FFI adapter), sized by the *_workspace_size
 *     queries.
 *
 * Return value: a ds_status.  Codes follow xla::ffi::ErrorCode (absl
 * numbering): DS_INVALID_ARGUMENT for the reference's shape errors (same
 * messages), DS_INTERNAL for CUDA errors (message = cudaGetErrorString).
 * ds_last_error() returns the calling thread's last message.
 */
#ifndef DS_B200_H_
#define DS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DS_API __attribute__((visibility("default")))
#else
#define DS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  DS_OK = 0,
  DS_INVALID_ARGUMENT = 3, /* xla::ffi::ErrorCode::kInvalidArgument */
  DS_INTERNAL = 13         /* xla::ffi::ErrorCode::kInternal */
};

/* A device tensor: data + dims[rank] (row-major, contiguous). */
typedef struct ds_buffer {
  void* data;
  const int64_t* dims;
  int64_t rank;
} ds_buffer;

/* Reduction bodies the DS pass rewrites (DsTransformPass.cpp:392-395). */
enum { DS_BODY_ADD = 0, DS_BODY_SUB = 1, DS_BODY_MUL = 2 };

/* dot_general algorithms. */
enum {
  /* exact integer-residue (Ozaki scheme II) GEMM on the int8 tcgen05 tensor
     cores; the default */
  DS_DOT_TENSOR_INT8 = 0,
  /* CUDA-core GEMM: exact f32 products (two_prod) summed in DS arithmetic */
  DS_DOT_CUDA_CORE = 1
};

/* dot_general dimension numbers, as stablehlo.dot_general's
   DotDimensionNumbers (lhs/rhs_batching_dimensions, lhs/rhs_contracting_
   dimensions): any batching dimensions, in any position, paired in list
   order; any number of contracting dimensions (none: an outer product),
   paired in list order; every other dimension is free.  The result is
   [batch (lhs order)..., lhs free (ascending)..., rhs free (ascending)...].
   Operands of rank up to DS_DOT_MAX_DIMS. */
#define DS_DOT_MAX_DIMS 8
typedef struct ds_dot_dims {
  int64_t n_batch;
  int64_t lhs_batch[DS_DOT_MAX_DIMS];
  int64_t rhs_batch[DS_DOT_MAX_DIMS];
  int64_t n_contracting;
  int64_t lhs_contracting[DS_DOT_MAX_DIMS];
  int64_t rhs_contracting[DS_DOT_MAX_DIMS];
} ds_dot_dims;

/* Message of the calling thread's last failing call ("" if none). */
DS_API const char* ds_last_error(void);

/* Library version string. */
DS_API const char* ds_version(void);

/* ---- split / recombine -------------------------------------------------- */

/* DsFromF64, cpp/ds_from_f64.cpp:18-49: x f64[...] -> y f32[..., 2],
   hi = f32(x), lo = f32(x - f64(hi)). */
DS_API int ds_from_f64(const ds_buffer* x, const ds_buffer* y, void* stream);

/* DsToF64, cpp/ds_to_f64.cpp:17-47: x f32[..., 2] -> y f64[...],
   y = f64(hi) + f64(lo). */
DS_API int ds_to_f64(const ds_buffer* x, const ds_buffer* y, void* stream);

/* ds_from_f32 ("Host" target, cpp/ds_from_f32.cpp:16-41): x f32[...] ->
   y f32[..., 2] = (x, 0). */
DS_API int ds_from_f32(const ds_buffer* x, const ds_buffer* y, void* stream);

/* ds_to_f32 ("Host" target, cpp/ds_to_f32.cpp:16-39): x f32[..., 2] ->
   y f32[...] = hi + lo (an f32 add). */
DS_API int ds_to_f32(const ds_buffer* x, const ds_buffer* y, void* stream);

/* ---- packed elementwise ------------------------------------------------- */

/* DsAdd, cpp/ds_add.cpp:23-73: a, b, y f32[..., 2]. */
DS_API int ds_add(const ds_buffer* a, const ds_buffer* b, const ds_buffer* y,
           void* stream);

/* DsSub, cpp/ds_sub.cpp:23-73. */
DS_API int ds_sub(const ds_buffer* a, const ds_buffer* b, const ds_buffer* y,
           void* stream);

/* DsMul, cpp/ds_mul.cpp:38-86 (Dekker two_prod with the 4097 split). */
DS_API int ds_mul(const ds_buffer* a, const ds_buffer* b, const ds_buffer* y,
           void* stream);

/* ---- fused f64 chains (rank-1 inputs of equal length) ------------------- */

/* DsFusedAddMul, cpp/ds_fused_add_mul.cpp:66-112: (x + y) * y,
   x, y f64[N] -> out f32[N, 2]. */
DS_API int ds_fused_add_mul(const ds_buffer* x, const ds_buffer* y,
                     const ds_buffer* out, void* stream);

/* DsFusedAddMulToF64, cpp/ds_fused_add_mul_to_f64.cpp:70-116: (x + y) * y,
   out f64[N]. */
DS_API int ds_fused_add_mul_to_f64(const ds_buffer* x, const ds_buffer* y,
                            const ds_buffer* out, void* stream);

/* DsFusedAxpy, cpp/ds_fused_axpy.cpp:75-120 (computes (x + y) * y, as the
   reference does; not built by the reference's CMakeLists). */
DS_API int ds_fused_axpy(const ds_buffer* x, const ds_buffer* y, const ds_buffer* out,
                  void* stream);

/* DsFusedAddMulToF64Cuda, cpp/ds_fused_add_mul_to_f64_cuda.cu:88-132. */
DS_API int ds_fused_add_mul_to_f64_cuda(const ds_buffer* x, const ds_buffer* y,
                                 const ds_buffer* out, void* stream);

/* DsFusedAddSubToF64Cuda, cpp/ds_fused_add_sub_to_f64_cuda.cu:52-121:
   (x + y) - x. */
DS_API int ds_fused_add_sub_to_f64_cuda(const ds_buffer* x, const ds_buffer* y,
                                 const ds_buffer* out, void* stream);

/* DsRecurrenceAddMulToF64Cuda, cpp/ds_recurrence_add_mul_to_f64_cuda.cu:
   98-149: z = split(x); k times z = (z + y) * y; out = f64(z).
   k < 0 -> DS_INVALID_ARGUMENT ("k must be nonnegative"). */
DS_API int ds_recurrence_add_mul_to_f64_cuda(const ds_buffer* x, const ds_buffer* y,
                                      int32_t k, const ds_buffer* out,
                                      void* stream);

/* Three-input (a + b) * c: DsFusedAddMulToF64 (cpp/ds_fused_add_mul_to_f64.
   cpp:81-93) with the multiplier split from its own input. */
DS_API int ds_fused_add_mul3_to_f64(const ds_buffer* a, const ds_buffer* b,
                             const ds_buffer* c, const ds_buffer* out,
                             void* stream);

/* x <- x * a + b, k times (ds_add(ds_mul(X, A), B)), the recurrence kernel
   (cpp/ds_recurrence_add_mul_to_f64_cuda.cu:69-93) with a multiply-add
   body. */
DS_API int ds_recurrence_mul_add_to_f64(const ds_buffer* x, const ds_buffer* a,
                                 const ds_buffer* b, int32_t k,
                                 const ds_buffer* out, void* stream);

/* ---- reduce (DsTransformPass.cpp:376-448) -------------------------------- */

/* DS reduce of SoA input (in_hi, in_lo f32[...]) over `dimensions` (which
   must be contiguous and ascending) with init (init_hi, init_lo: f32 rank-0
   device scalars) and body DS_BODY_*.  Outputs out_hi, out_lo have the input
   shape without the reduced dimensions.  The body is the pass's: acc =
   ds_op(acc, elem).  Elements are folded per thread in index order, then in
   a fixed shuffle/block tree, then block partials in block order, so results
   are deterministic for a given shape and device model (a full reduction
   uses up to 8 blocks per SM, so its order follows the SM count); init is
   applied once, last (subtract: init - sum; add: init + sum; multiply:
   init * product).
   The workspace (ds_reduce_workspace_size bytes) holds block partials: a
   full reduction needs it; a reduction over a leading dimension with few
   columns uses it to slice the reduced dimension across blocks (the slice
   count depends on the shape alone), and runs in one stage, in another
   order, when given less than ds_reduce_workspace_size bytes; other
   reductions need none. */
DS_API size_t ds_reduce_workspace_size(const ds_buffer* in, const int64_t* dimensions,
                                int64_t n_dimensions);
DS_API int ds_reduce(const ds_buffer* in_hi, const ds_buffer* in_lo,
              const ds_buffer* init_hi, const ds_buffer* init_lo,
              const int64_t* dimensions, int64_t n_dimensions, int32_t body,
              const ds_buffer* out_hi, const ds_buffer* out_lo,
              void* workspace, size_t workspace_bytes, void* stream);

/* The same with the pass's entry split and exit recombine fused: f64 input,
   f64 rank-0 init, f64 output (jnp.sum of an f64 array under the pass). */
DS_API int ds_reduce_f64(const ds_buffer* in, const ds_buffer* init,
                  const int64_t* dimensions, int64_t n_dimensions, int32_t body,
                  const ds_buffer* out, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ds_reduce_f64 for callers that cannot allocate device memory.  No
   counterpart in the reference.
   Some callers have no way to obtain scratch: an XLA-FFI handler bound
   without a scratch-allocator context, or code running next to a framework
   whose caching allocator (XLA's BFC allocator, torch's) has already reserved
   most of HBM, where a cudaMalloc of its own can fail and, because it may
   synchronise the device, would also stall every stream.  This entry point
   takes only inputs and outputs and allocates nothing: the partials that
   ds_reduce_f64 keeps in its workspace (the block partials of a full
   reduction, the slice partials of a reduction over a leading dimension
   with few columns) live in a library-owned static device array of 49152
   partials (384 KiB), which every GPU that loads the library holds until
   the process exits.  Results are bit-identical to ds_reduce_f64 given a
   workspace of ds_reduce_workspace_size bytes.
   - A reduction that would need more than 49152 partials returns
     DS_INVALID_ARGUMENT (full reductions use at most 8 per SM and sliced
     ones fewer than 49152, so this does not occur on B200).
   - The first call on each device looks up the array's device address
     (cudaGetSymbolAddress) with that device current; make that first call
     before any stream capture.
   - All calls share the array, which keeps the last call's contents (each
     call overwrites every slot it reads, so no clearing is needed); calls
     whose kernels overlap on the GPU race on it and must be ordered (same
     stream, or events). */
DS_API int ds_reduce_f64_noalloc(const ds_buffer* in, const ds_buffer* init,
                                 const int64_t* dimensions, int64_t n_dimensions,
                                 int32_t body, const ds_buffer* out,
                                 void* stream);

/* A variadic reduce (stablehlo.reduce with several inputs, which the
   reference pass leaves alone, DsTransformPass.cpp:377) whose body combines
   each input with its own add / subtract / multiply: n_inputs f64 tensors of
   one shape, each reduced over `dimensions` with bodies[k] and inits[k] into
   outs[k].  The reductions run one after another on the stream and share the
   workspace (ds_reduce_workspace_size of one input). */
DS_API int ds_reduce_f64_multi(const ds_buffer* const* ins, const ds_buffer* const* inits,
                               const int32_t* bodies, int32_t n_inputs,
                               const int64_t* dimensions, int64_t n_dimensions,
                               const ds_buffer* const* outs, void* workspace,
                               size_t workspace_bytes, void* stream);

/* DS reduce of a packed DS tensor in[..., 2] (the wire format of DsAdd and
   the other packed targets, cpp/ds_add.cpp:46-49) over `dimensions` of its
   logical shape in.dims[:-1]; init and result as in ds_reduce.  The
   workspace size is that of ds_reduce on the logical shape. */
DS_API int ds_reduce_packed(const ds_buffer* in, const ds_buffer* init_hi,
                            const ds_buffer* init_lo, const int64_t* dimensions,
                            int64_t n_dimensions, int32_t body,
                            const ds_buffer* out_hi, const ds_buffer* out_lo,
                            void* workspace, size_t workspace_bytes,
                            void* stream);

/* The split fused on input only: f64 input and rank-0 f64 init, SoA DS
   result (out_hi, out_lo) -- the pass's reduce of an f64 argument whose
   result stays in DS form (e.g. a partial sum that is combined further). */
DS_API int ds_reduce_from_f64(const ds_buffer* in, const ds_buffer* init,
                              const int64_t* dimensions, int64_t n_dimensions,
                              int32_t body, const ds_buffer* out_hi,
                              const ds_buffer* out_lo, void* workspace,
                              size_t workspace_bytes, void* stream);

/* ---- sharded reduce over the GPUs of one node ---------------------------- */

/* The reference reduces on one device (DsTransformPass.cpp:376-448); these
   entry points shard a full DS reduction of f64 data over one process per
   GPU.  Each rank owns one exchange buffer of ds_exchange_bytes() bytes
   (ds_exchange_alloc, which zeroes it and exports a CUDA IPC handle of
   ds_exchange_handle_bytes() bytes) and maps every other rank's buffer with
   ds_exchange_open.  Layout of a buffer: records[2][8] of 32 bytes at
   offset (parity * 8 + r) * 32 -- f32 hi, f32 lo, i64 n, u64 epoch, u64 pad
   -- and a sticky u32 error word at offset 512 (1 = a wait timed out). */
DS_API size_t ds_exchange_bytes(void);
DS_API size_t ds_exchange_handle_bytes(void);
DS_API int ds_exchange_alloc(void** buffer, void* handle);
DS_API int ds_exchange_open(const void* handle, void** buffer);
DS_API int ds_exchange_close(void* buffer);
DS_API int ds_exchange_free(void* buffer);
/* Reads the error word of this rank's own buffer (synchronous copy). */
DS_API int ds_exchange_error(const void* buffer, uint32_t* code);

/* Full DS reduction of this rank's f64 shard `in` (all dimensions), the
   ranks' DS totals exchanged through the exchange buffers, folded in rank
   order (ranks with empty shards skipped) and combined with the rank-0 f64
   init by `body`: every rank writes the same f64 bits to `out` (one
   element).  buffers[r] is rank r's exchange buffer as mapped in this
   process (buffers[rank] its own); world <= 8.  `epoch` numbers the calls
   1, 2, 3, ... in the same sequence on every rank.  A rank that waits more
   than timeout_ms for another writes NaN, sets the error word and returns
   (read it with ds_exchange_error); the exchange must then be rebuilt.
   Workspace: ds_reduce_f64_sharded_workspace_size(in) bytes, 8-byte
   aligned. */
DS_API size_t ds_reduce_f64_sharded_workspace_size(const ds_buffer* in);
DS_API int ds_reduce_f64_sharded(const ds_buffer* in, const ds_buffer* init, int32_t body,
                                 const ds_buffer* out, void* const* buffers, int32_t world,
                                 int32_t rank, uint64_t epoch, int32_t timeout_ms,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- dot_general (DsTransformPass.cpp:337-370) --------------------------- */

/* DS dot_general of SoA operands (lhs_hi, lhs_lo), (rhs_hi, rhs_lo) f32 with
   stablehlo dimension numbers (any batching, contracting and free
   dimensions, as the reference's handler clones them,
   DsTransformPass.cpp:345-356); result (out_hi, out_lo) f32 of shape
   [batch..., lhs free..., rhs free...].  The reference lowers this to four
   f32 dots (f32 accumulation) and a two_sum; here the product is computed
   from the exact DS values (see algorithm).  An operand whose batch, free or
   contracting dimensions do not nest into one stride each is first copied
   (one gather) into the workspace, which ds_dot_general_workspace_size
   counts; the contracting pairs are taken in whichever of their given
   order or the lhs or rhs dimension order needs the fewest copies. */
DS_API size_t ds_dot_general_workspace_size(const ds_buffer* lhs, const ds_buffer* rhs,
                                     const ds_dot_dims* dims, int32_t algorithm);
DS_API int ds_dot_general(const ds_buffer* lhs_hi, const ds_buffer* lhs_lo,
                   const ds_buffer* rhs_hi, const ds_buffer* rhs_lo,
                   const ds_dot_dims* dims, int32_t algorithm,
                   const ds_buffer* out_hi, const ds_buffer* out_lo,
                   void* workspace, size_t workspace_bytes, void* stream);

/* The same with split and recombine fused: f64 operands, f64 result (the
   pass on f64 arguments: emitFromFloat -> dot_general -> emitToFloat). */
DS_API int ds_dot_general_f64(const ds_buffer* lhs, const ds_buffer* rhs,
                       const ds_dot_dims* dims, int32_t algorithm,
                       const ds_buffer* out, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---- fused elementwise programs ----------------------------------------- */

/* The DS pass's lowering of an elementwise DAG (DsTransformPass.cpp:244-321:
   constants and f64 arguments split by emitFromFloat, broadcast_in_dim on hi
   and lo alike, add / subtract / multiply as DS operations, the result
   recombined at the return) run as ONE kernel per DAG.  `ops` lists the DAG
   in SSA order; operation j refers to earlier operations by index and the
   last one is the result:
     DS_FUSED_INPUT  a = input index (f64 inputs are split, f32 inputs become
                     (v, 0), packed inputs [..., 2] are DS pairs)
     DS_FUSED_CONST  value (split like an f64 argument)
     DS_FUSED_ADD / SUB / MUL  a, b
     DS_FUSED_NEG    a (exact: (-hi, -lo))
   Inputs broadcast to the output's logical shape with numpy's rules (packed
   tensors without their trailing 2).  The output is f64 (hi + lo in f64),
   f32 (hi + lo in f32, as ds_to_f32) or packed DS [..., 2].  The kernel is
   generated and compiled (NVRTC, sm_100a, no FMA contraction) on the first
   call for each program, types and shapes, then cached per device. */
enum { DS_FUSED_INPUT = 0, DS_FUSED_CONST = 1, DS_FUSED_ADD = 2, DS_FUSED_SUB = 3,
       DS_FUSED_MUL = 4, DS_FUSED_NEG = 5 };
enum { DS_FUSED_F64 = 0, DS_FUSED_F32 = 1, DS_FUSED_PACKED = 2 };
typedef struct ds_fused_op {
  int32_t code;
  int32_t a;
  int32_t b;
  int32_t reserved;
  double value;
} ds_fused_op;

DS_API int ds_fused_run(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                        const ds_buffer* const* inputs, int32_t n_inputs, int32_t out_type,
                        const ds_buffer* out, void* stream);
/* The generated CUDA source (for inspection); *len = its size + 1. */
DS_API int ds_fused_source(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                           const ds_buffer* const* inputs, int32_t n_inputs, int32_t out_type,
                           const ds_buffer* out, char* buf, size_t cap, size_t* len);
/* Generate and compile without loading (no GPU needed). */
DS_API int ds_fused_compile_check(const ds_fused_op* ops, int32_t n_ops,
                                  const int32_t* input_types, const ds_buffer* const* inputs,
                                  int32_t n_inputs, int32_t out_type, const ds_buffer* out);

/* A fused program reduced to one DS value: the program of ds_fused_run
   evaluated over every element of the logical shape `dims` (its inputs
   broadcast to it), and the results combined with `body` (DS_BODY_ADD or
   DS_BODY_MUL) and the init pair (0-d f32 device buffers, as ds_reduce).
   The result (out_hi, out_lo) is 0-d f32.  This is the pass's reduce
   (DsTransformPass.cpp:376-448) of an elementwise DAG (:282-321) without
   writing the DAG's values to memory.  Each thread folds the elements it
   visits; warp and block trees follow, and ds_reduce_packed combines the
   per-block partials with the init.  The order is fixed for a given size,
   so results are deterministic.  The workspace is 256-byte aligned and
   ds_fused_reduce_workspace_size bytes. */
DS_API size_t ds_fused_reduce_workspace_size(const int64_t* dims, int32_t rank);
DS_API int ds_fused_reduce(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                           const ds_buffer* const* inputs, int32_t n_inputs,
                           const int64_t* dims, int32_t rank, int32_t body,
                           const ds_buffer* init_hi, const ds_buffer* init_lo,
                           const ds_buffer* out_hi, const ds_buffer* out_lo,
                           void* workspace, size_t workspace_bytes, void* stream);
/* Generate and compile (NVRTC) the reduction kernel without running it. */
DS_API int ds_fused_reduce_compile_check(const ds_fused_op* ops, int32_t n_ops,
                                         const int32_t* input_types,
                                         const ds_buffer* const* inputs, int32_t n_inputs,
                                         const int64_t* dims, int32_t rank, int32_t body);

/* The same reduction over the trailing `n_reduced` dimensions of `dims`
   only: one DS value per row of the leading dimensions, written to
   out_hi / out_lo (f32, one element per row, row-major), each
   body(init, row total) -- the pass's reduce of an elementwise DAG over its
   last dimensions (DsTransformPass.cpp:376-448) without writing the DAG's
   values.  A block of 256 threads folds each row of at least 2048 values;
   shorter rows are folded by groups of 1-32 lanes (about eight values per
   lane), so the order is fixed per row length.  No workspace. */
DS_API int ds_fused_reduce_rows(const ds_fused_op* ops, int32_t n_ops,
                                const int32_t* input_types, const ds_buffer* const* inputs,
                                int32_t n_inputs, const int64_t* dims, int32_t rank,
                                int32_t n_reduced, int32_t body, const ds_buffer* init_hi,
                                const ds_buffer* init_lo, const ds_buffer* out_hi,
                                const ds_buffer* out_lo, void* stream);
/* Generate and compile (NVRTC) the per-row kernel without running it. */
DS_API int ds_fused_reduce_rows_compile_check(const ds_fused_op* ops, int32_t n_ops,
                                              const int32_t* input_types,
                                              const ds_buffer* const* inputs, int32_t n_inputs,
                                              const int64_t* dims, int32_t rank,
                                              int32_t n_reduced, int32_t body);

/* ---- diagnostics (no reference counterpart) ------------------------------ */

/* Per-kernel GPU time.  While enabled, each op brackets its main kernel with
   CUDA events on the launch stream under a family name ("elementwise",
   "recurrence", "reduce", "dot_simt", "dot_vec", "ozaki_split" (with its
   parts "ozaki_split_rows", "ozaki_split_rows_colmax", "ozaki_colmax" and
   "ozaki_split_cols"), "ozaki_gemm", "ozaki_crt", "ozaki_fix").
   ds_profile_read waits for the recorded events and returns the summed
   milliseconds and the launch count.  ds_profile_select limits the
   recording to the families named in a comma-separated list (NULL or ""
   records all), so that a timed loop pays for the brackets of one kernel
   only. */
/* Plan of the tensor-core dot_general for contraction length K: the number
   of int8 GEMMs (moduli) it runs and the bits each operand keeps relative to
   its row (column) maximum. */
DS_API int ds_dot_tensor_plan(int64_t K, int32_t* moduli, int32_t* bits);

/* Which tensor-core GEMM kernel the current device runs: *cta_pairs is the
   number of co-resident CTA pairs of the cta_group::2 kernel (0 when the
   one-CTA kernel is used), *query_error the CUDA error of the cluster
   occupancy query that decided it (0 if it succeeded). */
DS_API int ds_dot_tensor_kernel_info(int32_t* cta_pairs, int32_t* query_error);

DS_API void ds_profile_enable(int on);
DS_API void ds_profile_select(const char* names);
DS_API void ds_profile_reset(void);
DS_API int ds_profile_read(const char* name, double* total_ms, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* DS_B200_H_ */
