// Elementwise DS kernels: split/recombine, packed add/sub/mul, the fused f64
// chains and the two recurrences.
//
// Layout: f64 tensors are plain arrays; packed DS tensors are float2 arrays
// (hi, lo).  Each thread of the vector kernel handles a pair of consecutive
// elements per step with one 16-byte load per input (double2 for f64, float4
// for packed DS) and one 16-byte store, in a grid-stride loop sized to fill
// every SM; U pairs are loaded before any is computed so each thread keeps
// several loads in flight.  Unaligned views (an odd element offset) take the
// scalar kernel.  Everything is HBM-bound except the recurrences at large k.
#include "common.cuh"
#include "ds_arith.cuh"
#include "kernels.h"
#include "profile.h"

namespace dsb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;

template <class T> struct PairIO;

template <> struct PairIO<double> {
  static __device__ __forceinline__ void load(const double* p, int64_t i,
                                              double& x0, double& x1) {
    const double2 v = __ldcs(reinterpret_cast<const double2*>(p) + i);
    x0 = v.x;
    x1 = v.y;
  }
  static __device__ __forceinline__ void store(double* p, int64_t i, double x0,
                                               double x1) {
    __stcs(reinterpret_cast<double2*>(p) + i, make_double2(x0, x1));
  }
  static constexpr size_t kAlign = 16;
};

template <> struct PairIO<float2> {
  static __device__ __forceinline__ void load(const float2* p, int64_t i,
                                              float2& x0, float2& x1) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(p) + i);
    x0 = make_float2(v.x, v.y);
    x1 = make_float2(v.z, v.w);
  }
  static __device__ __forceinline__ void store(float2* p, int64_t i, float2 x0,
                                               float2 x1) {
    __stcs(reinterpret_cast<float4*>(p) + i, make_float4(x0.x, x0.y, x1.x, x1.y));
  }
  static constexpr size_t kAlign = 16;
};

template <> struct PairIO<float> {
  static __device__ __forceinline__ void load(const float* p, int64_t i,
                                              float& x0, float& x1) {
    const float2 v = __ldcs(reinterpret_cast<const float2*>(p) + i);
    x0 = v.x;
    x1 = v.y;
  }
  static __device__ __forceinline__ void store(float* p, int64_t i, float x0,
                                               float x1) {
    __stcs(reinterpret_cast<float2*>(p) + i, make_float2(x0, x1));
  }
  static constexpr size_t kAlign = 8;
};

__device__ __forceinline__ ds2 as_ds(float2 v) { return ds2{v.x, v.y}; }
__device__ __forceinline__ float2 as_f2(ds2 v) { return make_float2(v.hi, v.lo); }

// ---- element functors -----------------------------------------------------

struct OpFromF64 {
  __device__ float2 operator()(double x, double, double) const {
    return as_f2(from_f64(x));
  }
};
struct OpToF64 {
  __device__ double operator()(float2 x, float2, float2) const {
    return to_f64(as_ds(x));
  }
};
struct OpFromF32 {
  __device__ float2 operator()(float x, float, float) const {
    return make_float2(x, 0.0f);
  }
};
struct OpToF32 {
  __device__ float operator()(float2 x, float2, float2) const {
    return __fadd_rn(x.x, x.y);
  }
};
struct OpAdd {
  __device__ float2 operator()(float2 a, float2 b, float2) const {
    return as_f2(add(as_ds(a), as_ds(b)));
  }
};
struct OpSub {
  __device__ float2 operator()(float2 a, float2 b, float2) const {
    return as_f2(sub(as_ds(a), as_ds(b)));
  }
};
struct OpMul {
  __device__ float2 operator()(float2 a, float2 b, float2) const {
    return as_f2(mul(as_ds(a), as_ds(b)));
  }
};
// (x + y) * y, packed result (cpp/ds_fused_add_mul.cpp:88-101).
struct OpFusedAddMulPacked {
  __device__ float2 operator()(double x, double y, double) const {
    const ds2 X = from_f64(x), Y = from_f64(y);
    return as_f2(mul(add(X, Y), Y));
  }
};
// (x + y) * y -> f64 (cpp/ds_fused_add_mul_to_f64.cpp:81-93).
struct OpFusedAddMulF64 {
  __device__ double operator()(double x, double y, double) const {
    const ds2 X = from_f64(x), Y = from_f64(y);
    return to_f64(mul(add(X, Y), Y));
  }
};
// (x + y) - x -> f64 (cpp/ds_fused_add_sub_to_f64_cuda.cu:52-70).
struct OpFusedAddSubF64 {
  __device__ double operator()(double x, double y, double) const {
    const ds2 X = from_f64(x), Y = from_f64(y);
    return to_f64(sub(add(X, Y), X));
  }
};
// (a + b) * c -> f64.
struct OpFusedAddMul3F64 {
  __device__ double operator()(double a, double b, double c) const {
    return to_f64(mul(add(from_f64(a), from_f64(b)), from_f64(c)));
  }
};

// ---- generic vector / scalar kernels --------------------------------------

template <int NIN, class TIn, class TOut, class Op>
__global__ void __launch_bounds__(kThreads)
ew_pair_kernel(const TIn* __restrict__ a, const TIn* __restrict__ b,
               const TIn* __restrict__ c, TOut* __restrict__ out, int64_t n,
               Op op) {
  wait_previous_grid();  // launched as a programmatic dependent: the producer's writes
  const int64_t npairs = n >> 1;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       base < npairs; base += stride * kUnroll) {
    TIn a0[kUnroll], a1[kUnroll], b0[kUnroll], b1[kUnroll], c0[kUnroll], c1[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < npairs) {
        PairIO<TIn>::load(a, i, a0[u], a1[u]);
        if constexpr (NIN > 1) PairIO<TIn>::load(b, i, b0[u], b1[u]);
        if constexpr (NIN > 2) PairIO<TIn>::load(c, i, c0[u], c1[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < npairs) {
        PairIO<TOut>::store(out, i, op(a0[u], b0[u], c0[u]), op(a1[u], b1[u], c1[u]));
      }
    }
  }
  if ((n & 1) && blockIdx.x == 0 && threadIdx.x == 0) {
    const int64_t i = n - 1;
    TIn av = a[i], bv{}, cv{};
    if constexpr (NIN > 1) bv = b[i];
    if constexpr (NIN > 2) cv = c[i];
    out[i] = op(av, bv, cv);
  }
}

template <int NIN, class TIn, class TOut, class Op>
__global__ void __launch_bounds__(kThreads)
ew_scalar_kernel(const TIn* __restrict__ a, const TIn* __restrict__ b,
                 const TIn* __restrict__ c, TOut* __restrict__ out, int64_t n,
                 Op op) {
  wait_previous_grid();  // launched as a programmatic dependent: the producer's writes
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride) {
    TIn av = a[i], bv{}, cv{};
    if constexpr (NIN > 1) bv = b[i];
    if constexpr (NIN > 2) cv = c[i];
    out[i] = op(av, bv, cv);
  }
}

template <int NIN, class TIn, class TOut, class Op>
int launch_ew(const void* a, const void* b, const void* c, void* out, int64_t n,
              Op op, cudaStream_t s) {
  if (n <= 0) return ok();
  const TIn* ap = static_cast<const TIn*>(a);
  const TIn* bp = static_cast<const TIn*>(b);
  const TIn* cp = static_cast<const TIn*>(c);
  TOut* op_ = static_cast<TOut*>(out);
  bool vec = aligned(a, PairIO<TIn>::kAlign) && aligned(out, PairIO<TOut>::kAlign);
  if (NIN > 1) vec = vec && aligned(b, PairIO<TIn>::kAlign);
  if (NIN > 2) vec = vec && aligned(c, PairIO<TIn>::kAlign);
  // Programmatic dependent launches: a chain of calls on one stream overlaps
  // each launch with the previous kernel's tail (each kernel waits for its
  // predecessor before touching memory).
  ProfileScope prof("elementwise", s);
  if (vec) {
    const int64_t steps = ((n >> 1) + kUnroll - 1) / kUnroll;
    DSB_CUDA_TRY(launch_dependent(ew_pair_kernel<NIN, TIn, TOut, Op>,
                                  dim3(grid_for(steps, kThreads, 8)), dim3(kThreads), s, ap, bp,
                                  cp, op_, n, op));
  } else {
    DSB_CUDA_TRY(launch_dependent(ew_scalar_kernel<NIN, TIn, TOut, Op>,
                                  dim3(grid_for(n, kThreads, 8)), dim3(kThreads), s, ap, bp, cp,
                                  op_, n, op));
  }
  return launch_status();
}

// ---- recurrences ------------------------------------------------------------
//
// Each thread owns kChains elements and advances all of them one iteration at
// a time, so kChains independent DS dependency chains interleave in the
// pipeline.  The Veltkamp split of the loop-invariant multiplier is hoisted.
// The product's error term comes from one FMA wherever that equals Dekker's
// (fma_b_range / fma_p_range): one vote per iteration checks the warp's
// kChains products at once, so the common case is one straight-line block of
// about 36 f32 operations per element-iteration (ds_mul 14, ds_add 20, the
// range test about 2) instead of 45; a warp with any product out of range
// takes Dekker for those lanes.  The bits are Dekker's everywhere.  The outer
// loop is warp-uniform (lanes past n compute on zeros) so the vote sees the
// whole warp.

constexpr int kChains = 4;

// p = a.hi * b.hi for every chain and their exact errors, into p[] and e[].
__device__ __forceinline__ void head_products(const ds2 (&a)[kChains], const ds2 (&b)[kChains],
                                              const float (&bh)[kChains],
                                              const float (&bl)[kChains], bool b_ok,
                                              float (&p)[kChains], float (&e)[kChains]) {
  float lo = 0x1p127f, hi = 0.0f;
#pragma unroll
  for (int u = 0; u < kChains; ++u) {
    p[u] = __fmul_rn(a[u].hi, b[u].hi);
    lo = fminf(lo, fabsf(p[u]));
    hi = fmaxf(hi, fabsf(p[u]));
  }
  // fminf/fmaxf drop a NaN operand: a NaN product (a NaN a.hi; b_ok excludes
  // a NaN or infinite b) takes the FMA, whose error term is NaN as Dekker's is
  const bool ok = b_ok && lo >= 0x1p-90f && hi <= 0x1p110f;
  if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
    for (int u = 0; u < kChains; ++u) e[u] = __fmaf_rn(a[u].hi, b[u].hi, -p[u]);
  } else {
#pragma unroll
    for (int u = 0; u < kChains; ++u)
      e[u] = (b_ok && fma_p_range(p[u])) ? __fmaf_rn(a[u].hi, b[u].hi, -p[u])
                                         : dekker_err_bsplit(a[u].hi, bh[u], bl[u], p[u]);
  }
}

// z <- (z + y) * y, k times (cpp/ds_recurrence_add_mul_to_f64_cuda.cu:69-93).
__global__ void __launch_bounds__(kThreads)
recurrence_add_mul_kernel(const double* __restrict__ x, const double* __restrict__ y,
                          double* __restrict__ out, int64_t n, int32_t k) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       base - lane < n; base += stride * kChains) {
    ds2 z[kChains], Y[kChains];
    float yh[kChains], yl[kChains];
    bool y_ok = true;
#pragma unroll
    for (int u = 0; u < kChains; ++u) {
      const int64_t i = base + u * stride;
      const bool in = i < n;
      z[u] = from_f64(in ? x[i] : 0.0);
      Y[u] = from_f64(in ? y[i] : 0.0);
      split(Y[u].hi, yh[u], yl[u]);
      y_ok = y_ok && fma_b_range(Y[u].hi);
    }
    for (int32_t it = 0; it < k; ++it) {
      ds2 w[kChains];
      float p[kChains], e[kChains];
#pragma unroll
      for (int u = 0; u < kChains; ++u) w[u] = add(z[u], Y[u]);
      head_products(w, Y, yh, yl, y_ok, p, e);
#pragma unroll
      for (int u = 0; u < kChains; ++u) z[u] = mul_finish(w[u], Y[u], p[u], e[u]);
    }
#pragma unroll
    for (int u = 0; u < kChains; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) out[i] = to_f64(z[u]);
    }
  }
}

// x <- x * a + b, k times: ds_add(ds_mul(X, A), B).
__global__ void __launch_bounds__(kThreads)
recurrence_mul_add_kernel(const double* __restrict__ x, const double* __restrict__ a,
                          const double* __restrict__ b, double* __restrict__ out,
                          int64_t n, int32_t k) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       base - lane < n; base += stride * kChains) {
    ds2 z[kChains], A[kChains], B[kChains];
    float ah[kChains], al[kChains];
    bool a_ok = true;
#pragma unroll
    for (int u = 0; u < kChains; ++u) {
      const int64_t i = base + u * stride;
      const bool in = i < n;
      z[u] = from_f64(in ? x[i] : 0.0);
      A[u] = from_f64(in ? a[i] : 0.0);
      B[u] = from_f64(in ? b[i] : 0.0);
      split(A[u].hi, ah[u], al[u]);
      a_ok = a_ok && fma_b_range(A[u].hi);
    }
    for (int32_t it = 0; it < k; ++it) {
      float p[kChains], e[kChains];
      head_products(z, A, ah, al, a_ok, p, e);
#pragma unroll
      for (int u = 0; u < kChains; ++u) z[u] = add(mul_finish(z[u], A[u], p[u], e[u]), B[u]);
    }
#pragma unroll
    for (int u = 0; u < kChains; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) out[i] = to_f64(z[u]);
    }
  }
}

unsigned recurrence_grid(int64_t n, int32_t k) {
  // Streaming (small k): fill the machine like the other kernels.  Compute
  // bound (large k): one wave of full-occupancy blocks keeps every SM busy.
  const int64_t threads_needed = (n + kChains - 1) / kChains;
  return grid_for(threads_needed, kThreads, k > 4 ? 8 : 8);
}

}  // namespace

int ew_from_f64(const double* x, float* y, int64_t n, cudaStream_t s) {
  return launch_ew<1, double, float2>(x, nullptr, nullptr, y, n, OpFromF64{}, s);
}
int ew_to_f64(const float* x, double* y, int64_t n, cudaStream_t s) {
  return launch_ew<1, float2, double>(x, nullptr, nullptr, y, n, OpToF64{}, s);
}
int ew_from_f32(const float* x, float* y, int64_t n, cudaStream_t s) {
  return launch_ew<1, float, float2>(x, nullptr, nullptr, y, n, OpFromF32{}, s);
}
int ew_to_f32(const float* x, float* y, int64_t n, cudaStream_t s) {
  return launch_ew<1, float2, float>(x, nullptr, nullptr, y, n, OpToF32{}, s);
}
int ew_packed(int op, const float* a, const float* b, float* y, int64_t n,
              cudaStream_t s) {
  switch (op) {
    case 0: return launch_ew<2, float2, float2>(a, b, nullptr, y, n, OpAdd{}, s);
    case 1: return launch_ew<2, float2, float2>(a, b, nullptr, y, n, OpSub{}, s);
    default: return launch_ew<2, float2, float2>(a, b, nullptr, y, n, OpMul{}, s);
  }
}
int ew_fused_add_mul_packed(const double* x, const double* y, float* out, int64_t n,
                            cudaStream_t s) {
  return launch_ew<2, double, float2>(x, y, nullptr, out, n, OpFusedAddMulPacked{}, s);
}
int ew_fused_add_mul_f64(const double* x, const double* y, double* out, int64_t n,
                         cudaStream_t s) {
  return launch_ew<2, double, double>(x, y, nullptr, out, n, OpFusedAddMulF64{}, s);
}
int ew_fused_add_sub_f64(const double* x, const double* y, double* out, int64_t n,
                         cudaStream_t s) {
  return launch_ew<2, double, double>(x, y, nullptr, out, n, OpFusedAddSubF64{}, s);
}
int ew_fused_add_mul3_f64(const double* a, const double* b, const double* c,
                          double* out, int64_t n, cudaStream_t s) {
  return launch_ew<3, double, double>(a, b, c, out, n, OpFusedAddMul3F64{}, s);
}
int ew_recurrence_add_mul(const double* x, const double* y, double* out, int64_t n,
                          int32_t k, cudaStream_t s) {
  if (n <= 0) return ok();
  ProfileScope prof("recurrence", s);
  recurrence_add_mul_kernel<<<recurrence_grid(n, k), kThreads, 0, s>>>(x, y, out, n, k);
  return launch_status();
}
int ew_recurrence_mul_add(const double* x, const double* a, const double* b,
                          double* out, int64_t n, int32_t k, cudaStream_t s) {
  if (n <= 0) return ok();
  ProfileScope prof("recurrence", s);
  recurrence_mul_add_kernel<<<recurrence_grid(n, k), kThreads, 0, s>>>(x, a, b, out, n, k);
  return launch_status();
}

}  // namespace dsb
