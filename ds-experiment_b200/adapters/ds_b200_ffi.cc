// XLA-FFI handlers for libds_b200: the reference's custom-call targets
// (cpp/*.cpp and cpp/*.cu of rcast915/ds-experiment) re-pointed at the B200
// library, plus the new targets its retargeted DS pass emits (reduce,
// dot_general, fused elementwise regions).
//
// Built by adapters/CMakeLists.txt when the XLA-FFI headers are present
// (jax.ffi.include_dir()); this repository's image has no JAX, so here the
// same entry points are reached through ctypes (ds_b200/ffi.py).
//
// Every handler binds the platform stream (the reference's CUDA handlers
// launch on the legacy default stream and synchronise the device; these do
// neither) and forwards to one C-ABI entry point of include/ds_b200.h.  A
// status other than DS_OK becomes an ffi::Error with the same code (the C
// ABI numbers its codes as xla::ffi::ErrorCode) and the library's message.
// Scratch comes from XLA's allocator (ffi::ScratchAllocator).

#include <cuda_runtime.h>

#include <cstdint>
#include <optional>
#include <string>
#include <vector>

#include "ds_b200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

// A ds_buffer over an FFI buffer; owns its copy of the dimensions.
class View {
 public:
  template <typename Buf>
  explicit View(const Buf& buf) {
    auto d = buf.dimensions();
    dims_.assign(d.begin(), d.end());
    b_ = ds_buffer{const_cast<void*>(static_cast<const void*>(buf.untyped_data())),
                   dims_.data(), static_cast<int64_t>(dims_.size())};
  }
  View(const View&) = delete;
  View& operator=(const View&) = delete;
  const ds_buffer* get() const { return &b_; }

 private:
  std::vector<int64_t> dims_;
  ds_buffer b_{};
};

ffi::Error status(int st) {
  if (st == DS_OK) return ffi::Error::Success();
  return ffi::Error(static_cast<ffi::ErrorCode>(st), std::string(ds_last_error()));
}

// Scratch of `bytes` (at least 1) from XLA, 256-byte aligned.
std::optional<void*> scratch(ffi::ScratchAllocator& alloc, size_t bytes) {
  return alloc.Allocate(bytes ? bytes : 1, 256);
}

ffi::Error no_scratch(const char* what) {
  return ffi::Error(ffi::ErrorCode::kResourceExhausted, std::string(what) + ": no scratch");
}

template <typename T>
std::vector<T> to_vector(ffi::Span<const T> s) {
  return std::vector<T>(s.begin(), s.end());
}

}  // namespace

// ---- split / recombine (cpp/ds_from_f64.cpp:18-49, ds_to_f64.cpp:17-47,
//      ds_from_f32.cpp:16-41, ds_to_f32.cpp:16-39) -----------------------------

static ffi::Error DsFromF64Impl(cudaStream_t s, ffi::Buffer<ffi::F64> x,
                                ffi::ResultBuffer<ffi::F32> y) {
  View X(x), Y(*y);
  return status(ds_from_f64(X.get(), Y.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsFromF64, DsFromF64Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

static ffi::Error DsToF64Impl(cudaStream_t s, ffi::Buffer<ffi::F32> x,
                              ffi::ResultBuffer<ffi::F64> y) {
  View X(x), Y(*y);
  return status(ds_to_f64(X.get(), Y.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsToF64, DsToF64Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F64>>());

// The reference registers ds_from_f32 / ds_to_f32 for the "Host" platform;
// these run on the GPU and are registered for "CUDA".
static ffi::Error DsFromF32Impl(cudaStream_t s, ffi::Buffer<ffi::F32> x,
                                ffi::ResultBuffer<ffi::F32> y) {
  View X(x), Y(*y);
  return status(ds_from_f32(X.get(), Y.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsFromF32, DsFromF32Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());
XLA_FFI_REGISTER_HANDLER(ffi::GetXlaFfiApi(), "ds_from_f32", "CUDA", DsFromF32);

static ffi::Error DsToF32Impl(cudaStream_t s, ffi::Buffer<ffi::F32> x,
                              ffi::ResultBuffer<ffi::F32> y) {
  View X(x), Y(*y);
  return status(ds_to_f32(X.get(), Y.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsToF32, DsToF32Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());
XLA_FFI_REGISTER_HANDLER(ffi::GetXlaFfiApi(), "ds_to_f32", "CUDA", DsToF32);

// ---- packed elementwise (cpp/ds_add.cpp:67-73, ds_sub.cpp:67-73,
//      ds_mul.cpp:80-86) ----------------------------------------------------------

#define DS_PACKED_HANDLER(Symbol, fn)                                                     \
  static ffi::Error Symbol##Impl(cudaStream_t s, ffi::Buffer<ffi::F32> a,               \
                                 ffi::Buffer<ffi::F32> b, ffi::ResultBuffer<ffi::F32> y) { \
    View A(a), B(b), Y(*y);                                                               \
    return status(fn(A.get(), B.get(), Y.get(), s));                                      \
  }                                                                                       \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(Symbol, Symbol##Impl,                                     \
                                ffi::Ffi::Bind()                                          \
                                    .Ctx<ffi::PlatformStream<cudaStream_t>>()             \
                                    .Arg<ffi::Buffer<ffi::F32>>()                         \
                                    .Arg<ffi::Buffer<ffi::F32>>()                         \
                                    .Ret<ffi::Buffer<ffi::F32>>());

DS_PACKED_HANDLER(DsAdd, ds_add)
DS_PACKED_HANDLER(DsSub, ds_sub)
DS_PACKED_HANDLER(DsMul, ds_mul)

// ---- fused f64 chains (cpp/ds_fused_add_mul.cpp:106-112,
//      ds_fused_add_mul_to_f64.cpp:110-116, ds_fused_axpy.cpp:114-120,
//      ds_fused_add_mul_to_f64_cuda.cu:126-132,
//      ds_fused_add_sub_to_f64_cuda.cu:115-121) ------------------------------------

static ffi::Error DsFusedAddMulImpl(cudaStream_t s, ffi::Buffer<ffi::F64> x,
                                    ffi::Buffer<ffi::F64> y, ffi::ResultBuffer<ffi::F32> out) {
  View X(x), Y(y), O(*out);
  return status(ds_fused_add_mul(X.get(), Y.get(), O.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsFusedAddMul, DsFusedAddMulImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

#define DS_CHAIN_HANDLER(Symbol, fn)                                                      \
  static ffi::Error Symbol##Impl(cudaStream_t s, ffi::Buffer<ffi::F64> x,               \
                                 ffi::Buffer<ffi::F64> y, ffi::ResultBuffer<ffi::F64> out) { \
    View X(x), Y(y), O(*out);                                                             \
    return status(fn(X.get(), Y.get(), O.get(), s));                                     \
  }                                                                                       \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(Symbol, Symbol##Impl,                                     \
                                ffi::Ffi::Bind()                                          \
                                    .Ctx<ffi::PlatformStream<cudaStream_t>>()             \
                                    .Arg<ffi::Buffer<ffi::F64>>()                         \
                                    .Arg<ffi::Buffer<ffi::F64>>()                         \
                                    .Ret<ffi::Buffer<ffi::F64>>());

DS_CHAIN_HANDLER(DsFusedAddMulToF64, ds_fused_add_mul_to_f64)
DS_CHAIN_HANDLER(DsFusedAxpy, ds_fused_axpy)
DS_CHAIN_HANDLER(DsFusedAddMulToF64Cuda, ds_fused_add_mul_to_f64_cuda)
DS_CHAIN_HANDLER(DsFusedAddSubToF64Cuda, ds_fused_add_sub_to_f64_cuda)

// (a + b) * c on three f64 inputs.
static ffi::Error DsFusedAddMul3ToF64Impl(cudaStream_t s, ffi::Buffer<ffi::F64> a,
                                          ffi::Buffer<ffi::F64> b, ffi::Buffer<ffi::F64> c,
                                          ffi::ResultBuffer<ffi::F64> out) {
  View A(a), B(b), C(c), O(*out);
  return status(ds_fused_add_mul3_to_f64(A.get(), B.get(), C.get(), O.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsFusedAddMul3ToF64, DsFusedAddMul3ToF64Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Ret<ffi::Buffer<ffi::F64>>());

// ---- recurrences (cpp/ds_recurrence_add_mul_to_f64_cuda.cu:142-149) -----------

static ffi::Error DsRecurrenceAddMulToF64CudaImpl(cudaStream_t s, ffi::Buffer<ffi::F64> x,
                                                  ffi::Buffer<ffi::F64> y, int32_t k,
                                                  ffi::ResultBuffer<ffi::F64> out) {
  View X(x), Y(y), O(*out);
  return status(ds_recurrence_add_mul_to_f64_cuda(X.get(), Y.get(), k, O.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsRecurrenceAddMulToF64Cuda, DsRecurrenceAddMulToF64CudaImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Attr<int32_t>("k")
                                  .Ret<ffi::Buffer<ffi::F64>>());

static ffi::Error DsRecurrenceMulAddToF64Impl(cudaStream_t s, ffi::Buffer<ffi::F64> x,
                                              ffi::Buffer<ffi::F64> a, ffi::Buffer<ffi::F64> b,
                                              int32_t k, ffi::ResultBuffer<ffi::F64> out) {
  View X(x), A(a), B(b), O(*out);
  return status(ds_recurrence_mul_add_to_f64(X.get(), A.get(), B.get(), k, O.get(), s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsRecurrenceMulAddToF64, DsRecurrenceMulAddToF64Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Attr<int32_t>("k")
                                  .Ret<ffi::Buffer<ffi::F64>>());

// ---- reduce (the pass's reduce rewrite, DsTransformPass.cpp:376-448) -----------

// SoA DS input (hi, lo) and init pair -> (hi, lo).
static ffi::Error DsReduceImpl(cudaStream_t s, ffi::ScratchAllocator alloc,
                               ffi::Buffer<ffi::F32> hi, ffi::Buffer<ffi::F32> lo,
                               ffi::Buffer<ffi::F32> init_hi, ffi::Buffer<ffi::F32> init_lo,
                               ffi::Span<const int64_t> dimensions, int32_t body,
                               ffi::ResultBuffer<ffi::F32> out_hi,
                               ffi::ResultBuffer<ffi::F32> out_lo) {
  View H(hi), L(lo), IH(init_hi), IL(init_lo), OH(*out_hi), OL(*out_lo);
  const std::vector<int64_t> dims = to_vector(dimensions);
  const size_t need = ds_reduce_workspace_size(H.get(), dims.data(), dims.size());
  auto ws = scratch(alloc, need);
  if (!ws) return no_scratch("ds_reduce");
  return status(ds_reduce(H.get(), L.get(), IH.get(), IL.get(), dims.data(), dims.size(), body,
                          OH.get(), OL.get(), *ws, need, s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsReduce, DsReduceImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<ffi::Span<const int64_t>>("dimensions")
                                  .Attr<int32_t>("body")
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

// Packed DS input [..., 2] (the wire format of DsAdd) -> (hi, lo).
static ffi::Error DsReducePackedImpl(cudaStream_t s, ffi::ScratchAllocator alloc,
                                     ffi::Buffer<ffi::F32> x, ffi::Buffer<ffi::F32> init_hi,
                                     ffi::Buffer<ffi::F32> init_lo,
                                     ffi::Span<const int64_t> dimensions, int32_t body,
                                     ffi::ResultBuffer<ffi::F32> out_hi,
                                     ffi::ResultBuffer<ffi::F32> out_lo) {
  View X(x), IH(init_hi), IL(init_lo), OH(*out_hi), OL(*out_lo);
  const std::vector<int64_t> dims = to_vector(dimensions);
  // sized on the logical shape, without the trailing 2
  std::vector<int64_t> logical(X.get()->dims, X.get()->dims + X.get()->rank - 1);
  ds_buffer lb{X.get()->data, logical.data(), static_cast<int64_t>(logical.size())};
  const size_t need = ds_reduce_workspace_size(&lb, dims.data(), dims.size());
  auto ws = scratch(alloc, need);
  if (!ws) return no_scratch("ds_reduce_packed");
  return status(ds_reduce_packed(X.get(), IH.get(), IL.get(), dims.data(), dims.size(), body,
                                 OH.get(), OL.get(), *ws, need, s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsReducePacked, DsReducePackedImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<ffi::Span<const int64_t>>("dimensions")
                                  .Attr<int32_t>("body")
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

// f64 input and init -> f64 (split and recombine fused): what the retargeted
// pass emits for a reduce of f64 values.
static ffi::Error DsReduceF64Impl(cudaStream_t s, ffi::ScratchAllocator alloc,
                                  ffi::Buffer<ffi::F64> x, ffi::Buffer<ffi::F64> init,
                                  ffi::Span<const int64_t> dimensions, int32_t body,
                                  ffi::ResultBuffer<ffi::F64> out) {
  View X(x), I(init), O(*out);
  const std::vector<int64_t> dims = to_vector(dimensions);
  const size_t need = ds_reduce_workspace_size(X.get(), dims.data(), dims.size());
  auto ws = scratch(alloc, need);
  if (!ws) return no_scratch("ds_reduce_f64");
  return status(ds_reduce_f64(X.get(), I.get(), dims.data(), dims.size(), body, O.get(), *ws,
                              need, s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsReduceF64, DsReduceF64Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Attr<ffi::Span<const int64_t>>("dimensions")
                                  .Attr<int32_t>("body")
                                  .Ret<ffi::Buffer<ffi::F64>>());

// ---- dot_general (the pass's dot_general rewrite, DsTransformPass.cpp:337-370)

namespace {

bool dot_dims(ffi::Span<const int64_t> lb, ffi::Span<const int64_t> rb,
              ffi::Span<const int64_t> lc, ffi::Span<const int64_t> rc, ds_dot_dims& d) {
  if (lb.size() != rb.size() || lc.size() != rc.size() || lb.size() > DS_DOT_MAX_DIMS ||
      lc.size() > DS_DOT_MAX_DIMS)
    return false;
  d = ds_dot_dims{};
  d.n_batch = static_cast<int64_t>(lb.size());
  for (size_t i = 0; i < lb.size(); ++i) {
    d.lhs_batch[i] = lb[i];
    d.rhs_batch[i] = rb[i];
  }
  d.n_contracting = static_cast<int64_t>(lc.size());
  for (size_t i = 0; i < lc.size(); ++i) {
    d.lhs_contracting[i] = lc[i];
    d.rhs_contracting[i] = rc[i];
  }
  return true;
}

ffi::Error bad_dot_dims() {
  return ffi::Error(ffi::ErrorCode::kInvalidArgument,
                    "dot_general: mismatched or too many dimension numbers");
}

}  // namespace

static ffi::Error DsDotGeneralImpl(cudaStream_t s, ffi::ScratchAllocator alloc,
                                   ffi::Buffer<ffi::F32> a_hi, ffi::Buffer<ffi::F32> a_lo,
                                   ffi::Buffer<ffi::F32> b_hi, ffi::Buffer<ffi::F32> b_lo,
                                   ffi::Span<const int64_t> lhs_batch,
                                   ffi::Span<const int64_t> rhs_batch,
                                   ffi::Span<const int64_t> lhs_contracting,
                                   ffi::Span<const int64_t> rhs_contracting, int32_t algorithm,
                                   ffi::ResultBuffer<ffi::F32> out_hi,
                                   ffi::ResultBuffer<ffi::F32> out_lo) {
  ds_dot_dims d;
  if (!dot_dims(lhs_batch, rhs_batch, lhs_contracting, rhs_contracting, d)) return bad_dot_dims();
  View AH(a_hi), AL(a_lo), BH(b_hi), BL(b_lo), OH(*out_hi), OL(*out_lo);
  const size_t need = ds_dot_general_workspace_size(AH.get(), BH.get(), &d, algorithm);
  auto ws = scratch(alloc, need);
  if (!ws) return no_scratch("ds_dot_general");
  return status(ds_dot_general(AH.get(), AL.get(), BH.get(), BL.get(), &d, algorithm, OH.get(),
                               OL.get(), *ws, need, s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsDotGeneral, DsDotGeneralImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<ffi::Span<const int64_t>>("lhs_batching_dimensions")
                                  .Attr<ffi::Span<const int64_t>>("rhs_batching_dimensions")
                                  .Attr<ffi::Span<const int64_t>>("lhs_contracting_dimensions")
                                  .Attr<ffi::Span<const int64_t>>("rhs_contracting_dimensions")
                                  .Attr<int32_t>("algorithm")
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

static ffi::Error DsDotGeneralF64Impl(cudaStream_t s, ffi::ScratchAllocator alloc,
                                      ffi::Buffer<ffi::F64> a, ffi::Buffer<ffi::F64> b,
                                      ffi::Span<const int64_t> lhs_batch,
                                      ffi::Span<const int64_t> rhs_batch,
                                      ffi::Span<const int64_t> lhs_contracting,
                                      ffi::Span<const int64_t> rhs_contracting,
                                      int32_t algorithm, ffi::ResultBuffer<ffi::F64> out) {
  ds_dot_dims d;
  if (!dot_dims(lhs_batch, rhs_batch, lhs_contracting, rhs_contracting, d)) return bad_dot_dims();
  View A(a), B(b), O(*out);
  const size_t need = ds_dot_general_workspace_size(A.get(), B.get(), &d, algorithm);
  auto ws = scratch(alloc, need);
  if (!ws) return no_scratch("ds_dot_general_f64");
  return status(ds_dot_general_f64(A.get(), B.get(), &d, algorithm, O.get(), *ws, need, s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsDotGeneralF64, DsDotGeneralF64Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Arg<ffi::Buffer<ffi::F64>>()
                                  .Attr<ffi::Span<const int64_t>>("lhs_batching_dimensions")
                                  .Attr<ffi::Span<const int64_t>>("rhs_batching_dimensions")
                                  .Attr<ffi::Span<const int64_t>>("lhs_contracting_dimensions")
                                  .Attr<ffi::Span<const int64_t>>("rhs_contracting_dimensions")
                                  .Attr<int32_t>("algorithm")
                                  .Ret<ffi::Buffer<ffi::F64>>());

// ---- fused elementwise regions (one kernel per region) --------------------------
//
// The region travels as data: per operation a code (DS_FUSED_*), two operand
// indices and a constant, as four arrays of the custom call's backend_config;
// input_types gives each input's kind (DS_FUSED_F64 / F32 / PACKED) and
// out_type the result's.  The inputs are the call's operands, in order.

namespace {

bool fused_program(ffi::Span<const int32_t> codes, ffi::Span<const int32_t> a,
                   ffi::Span<const int32_t> b, ffi::Span<const double> values,
                   std::vector<ds_fused_op>& ops) {
  const size_t n = codes.size();
  if (a.size() != n || b.size() != n || values.size() != n) return false;
  ops.resize(n);
  for (size_t i = 0; i < n; ++i) ops[i] = ds_fused_op{codes[i], a[i], b[i], 0, values[i]};
  return true;
}

}  // namespace

static ffi::Error DsFusedImpl(cudaStream_t s, ffi::RemainingArgs args,
                              ffi::Span<const int32_t> codes, ffi::Span<const int32_t> a,
                              ffi::Span<const int32_t> b, ffi::Span<const double> values,
                              ffi::Span<const int32_t> input_types, int32_t out_type,
                              ffi::Result<ffi::AnyBuffer> out) {
  std::vector<ds_fused_op> ops;
  if (!fused_program(codes, a, b, values, ops) || input_types.size() != args.size())
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "ds_fused: malformed program");
  std::vector<std::vector<int64_t>> dims(args.size());
  std::vector<ds_buffer> bufs(args.size());
  std::vector<const ds_buffer*> ptrs(args.size());
  for (size_t i = 0; i < args.size(); ++i) {
    auto arg = args.get<ffi::AnyBuffer>(i);
    if (arg.has_error()) return arg.error();
    auto d = arg->dimensions();
    dims[i].assign(d.begin(), d.end());
    bufs[i] = ds_buffer{arg->untyped_data(), dims[i].data(), static_cast<int64_t>(dims[i].size())};
    ptrs[i] = &bufs[i];
  }
  const std::vector<int32_t> types = to_vector(input_types);
  View O(*out);
  return status(ds_fused_run(ops.data(), static_cast<int32_t>(ops.size()), types.data(),
                             ptrs.data(), static_cast<int32_t>(ptrs.size()), out_type, O.get(),
                             s));
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(DsFused, DsFusedImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .RemainingArgs()
                                  .Attr<ffi::Span<const int32_t>>("codes")
                                  .Attr<ffi::Span<const int32_t>>("a")
                                  .Attr<ffi::Span<const int32_t>>("b")
                                  .Attr<ffi::Span<const double>>("values")
                                  .Attr<ffi::Span<const int32_t>>("input_types")
                                  .Attr<int32_t>("out_type")
                                  .Ret<ffi::AnyBuffer>());
