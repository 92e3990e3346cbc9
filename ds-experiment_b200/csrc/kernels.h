// Internal launchers of libds_b200 (device pointers, caller's stream; no
// shape checks -- the C ABI in capi.cpp validates before calling these).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace dsb {

// elementwise.cu
int ew_from_f64(const double* x, float* y, int64_t n, cudaStream_t s);
int ew_to_f64(const float* x, double* y, int64_t n, cudaStream_t s);
int ew_from_f32(const float* x, float* y, int64_t n, cudaStream_t s);
int ew_to_f32(const float* x, float* y, int64_t n, cudaStream_t s);
int ew_packed(int op, const float* a, const float* b, float* y, int64_t n, cudaStream_t s);
int ew_fused_add_mul_packed(const double* x, const double* y, float* out, int64_t n,
                            cudaStream_t s);
int ew_fused_add_mul_f64(const double* x, const double* y, double* out, int64_t n,
                         cudaStream_t s);
int ew_fused_add_sub_f64(const double* x, const double* y, double* out, int64_t n,
                         cudaStream_t s);
int ew_fused_add_mul3_f64(const double* a, const double* b, const double* c, double* out,
                          int64_t n, cudaStream_t s);
int ew_recurrence_add_mul(const double* x, const double* y, double* out, int64_t n,
                          int32_t k, cudaStream_t s);
int ew_recurrence_mul_add(const double* x, const double* a, const double* b, double* out,
                          int64_t n, int32_t k, cudaStream_t s);

// layout.cu: dst (contiguous, row-major over size[0..nd)) = src at offsets
// sum_d index_d * stride[d] (elements of elem_bytes = 4 or 8); unit sizes
// are skipped, at most kGatherMaxDims others.
constexpr int kGatherMaxDims = 8;
int gather_strided(const void* src, void* dst, int elem_bytes, const int64_t* size,
                   const int64_t* stride, int nd, cudaStream_t s);

// reduce.cu
struct ReduceArgs {
  const double* in_f64 = nullptr;  // either f64 input ...
  const float* in_hi = nullptr;    // ... or SoA DS input ...
  const float* in_lo = nullptr;
  const float* in_packed = nullptr;  // ... or packed DS input [..., 2]
  const double* init_f64 = nullptr;  // rank-0 init (f64, or hi/lo)
  const float* init_hi = nullptr;
  const float* init_lo = nullptr;
  double* out_f64 = nullptr;  // either f64 output ...
  float* out_hi = nullptr;    // ... or SoA DS output
  float* out_lo = nullptr;
  int64_t outer = 1, red = 0, inner = 1;
  int body = 0;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
};
size_t reduce_workspace_bytes(int64_t outer, int64_t red, int64_t inner);
int reduce_launch(const ReduceArgs& a, cudaStream_t s);
// The same with the full-reduction partials in a static device array.
int reduce_launch_noalloc(ReduceArgs a, cudaStream_t s);

// Sharded full reduction of f64 shards, one per rank, with the DS totals
// exchanged through peer-mapped exchange buffers (layout in reduce.cu).
constexpr int kExchangeMaxRanks = 8;
constexpr size_t kExchangeBytes = 1024;
constexpr size_t kExchangeErrorOffset = 512;
struct ShardedReduceArgs {
  const double* in = nullptr;
  int64_t n = 0;
  const double* init = nullptr;
  double* out = nullptr;
  int body = 0;
  void* const* buffers = nullptr;  // host array: rank r's exchange buffer, as mapped here
  int world = 1, rank = 0;
  uint64_t epoch = 1;
  int64_t timeout_ns = 1000000000;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
};
size_t reduce_sharded_workspace_bytes(int64_t n);
int reduce_sharded_launch(const ShardedReduceArgs& a, cudaStream_t s);

// peer.cu: exchange buffers shared between processes (CUDA IPC).
size_t peer_handle_bytes();
int peer_alloc(size_t bytes, void** buf, void* handle);
int peer_open(const void* handle, void** buf);
int peer_close(void* buf);
int peer_free(void* buf);
int peer_read_error(const void* buf, uint32_t* code);

// Operand of a dot: element (b, r, k) of a batched [batch, rows, K] view at
// base[b * s_b + r * s_r + k * s_k], given as f64 or as SoA hi/lo f32.
struct DotOperand {
  const double* f64 = nullptr;
  const float* hi = nullptr;
  const float* lo = nullptr;
  int64_t s_b = 0, s_r = 0, s_k = 0;
};
// Result element (b, i, j) at base[b * M * N + i * N + j].
struct DotResult {
  double* f64 = nullptr;
  float* hi = nullptr;
  float* lo = nullptr;
};
struct DotProblem {
  DotOperand a;  // rows = M
  DotOperand b;  // rows = N (B^T view)
  DotResult c;
  int64_t batch = 1, M = 0, N = 0, K = 0;
};

// dot_simt.cu: CUDA-core GEMM with exact products and DS accumulation.
int dot_simt(const DotProblem& p, cudaStream_t s);
// dot_simt.cu: batched vector dot products (M == N == 1), HBM-bound.
size_t dot_vec_workspace_bytes(int64_t batch, int64_t K);
int dot_batched_vec(const DotProblem& p, void* workspace, size_t workspace_bytes,
                    cudaStream_t s);

// dot_ozaki.cu: int8 tensor-core Ozaki-II GEMM.
size_t dot_ozaki_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K);
bool dot_ozaki_supported(int64_t M, int64_t N, int64_t K);
int dot_ozaki_params(int64_t K, int* moduli, int* bits);
int dot_ozaki_kernel_info(int* cta_pairs, int* query_error);
int dot_ozaki(const DotProblem& p, void* workspace, size_t workspace_bytes, cudaStream_t s);

}  // namespace dsb
