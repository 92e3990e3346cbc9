// CUDA-core DS dot_general.
//
// Every multiply-accumulate takes the exact DS operands a = ah + al and
// b = bh + bl, forms the exact leading product p + e = ah * bh (p = fl(ah*bh),
// e = fma(ah, bh, -p)), adds the cross terms ah*bl + al*bh + al*bl into e with
// FMAs, and accumulates p into a DS pair with Knuth's two_sum followed by a
// fast two_sum renormalisation, so every step rounds at the DS level
// (~2^-48 of the running sum) -- far below the reference's f32-accumulated
// sub-dots (DsTransformPass.cpp:359-365).  16 FP32-pipe instructions per MAC.
//
// GEMM: 64x64 output tile per 256-thread block, 4x4 outputs per thread, K
// staged through shared memory 16 at a time as hi/lo planes.  Operands are
// generic strided views, read coalesced along whichever of (row, k) has
// stride 1.  Batched vector dots (M = N = 1) stream both operands once
// (16 bytes per MAC for f64 inputs), split K over several blocks when the
// batch is small, and fold block partials in a fixed order.
#include "common.cuh"
#include "ds_arith.cuh"
#include "kernels.h"
#include "profile.h"

namespace dsb {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, kThreads = 256;

struct Acc {
  float s, c;
};

// (s, c) += a * b with a = (ah, al), b = (bh, bl); (s, c) is renormalised
// after every step (fast two_sum), so |c| stays below ulp(s) and its own
// rounding errors stay at the DS level (~2^-48 |s|) instead of growing with K.
__device__ __forceinline__ void mac(Acc& acc, float ah, float al, float bh, float bl) {
  const float p = __fmul_rn(ah, bh);
  float t = __fmaf_rn(ah, bh, -p);
  t = __fmaf_rn(ah, bl, t);
  t = __fmaf_rn(al, bh, t);
  t = __fmaf_rn(al, bl, t);
  float s, e;
  two_sum(acc.s, p, s, e);
  const float c = __fadd_rn(acc.c, __fadd_rn(e, t));
  acc.s = __fadd_rn(s, c);
  acc.c = __fsub_rn(c, __fsub_rn(acc.s, s));
}

__device__ __forceinline__ Acc acc_merge(Acc x, Acc y) {
  float s, e;
  two_sum(x.s, y.s, s, e);
  return Acc{s, __fadd_rn(__fadd_rn(x.c, y.c), e)};
}

// Renormalise (s, c) into a DS pair (fast two_sum; |c| is small against s).
__device__ __forceinline__ ds2 acc_final(Acc a) {
  const float hi = __fadd_rn(a.s, a.c);
  const float lo = __fsub_rn(a.c, __fsub_rn(hi, a.s));
  return ds2{hi, lo};
}

__device__ __forceinline__ ds2 load_ds(const DotOperand& o, int64_t idx) {
  return o.f64 ? from_f64(o.f64[idx]) : ds2{o.hi[idx], o.lo[idx]};
}

__device__ __forceinline__ void store_result(const DotResult& c, int64_t idx, ds2 v) {
  if (c.f64) {
    c.f64[idx] = to_f64(v);
  } else {
    c.hi[idx] = v.hi;
    c.lo[idx] = v.lo;
  }
}

// Stage one BK x BROWS tile of an operand into (hi, lo) shared planes.
template <int BROWS>
__device__ __forceinline__ void stage(const DotOperand& o, int64_t b, int64_t row0,
                                      int64_t k0, int64_t rows, int64_t K,
                                      float (*sh)[BROWS + 4], float (*sl)[BROWS + 4]) {
  constexpr int kElems = BROWS * BK / kThreads;
  const bool k_fast = o.s_k == 1;
#pragma unroll
  for (int q = 0; q < kElems; ++q) {
    const int e = threadIdx.x + q * kThreads;
    const int kk = k_fast ? (e % BK) : (e / BROWS);
    const int rr = k_fast ? (e / BK) : (e % BROWS);
    const int64_t r = row0 + rr, k = k0 + kk;
    ds2 v{0.0f, 0.0f};
    if (r < rows && k < K) v = load_ds(o, b * o.s_b + r * o.s_r + k * o.s_k);
    sh[kk][rr] = v.hi;
    sl[kk][rr] = v.lo;
  }
}

__global__ void __launch_bounds__(kThreads)
gemm_simt_kernel(DotProblem p) {
  __shared__ float ah_s[BK][BM + 4], al_s[BK][BM + 4];
  __shared__ float bh_s[BK][BN + 4], bl_s[BK][BN + 4];
  const int64_t b = blockIdx.z;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  Acc acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = Acc{0.0f, 0.0f};

  for (int64_t k0 = 0; k0 < p.K; k0 += BK) {
    stage<BM>(p.a, b, m0, k0, p.M, p.K, ah_s, al_s);
    stage<BN>(p.b, b, n0, k0, p.N, p.K, bh_s, bl_s);
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < BK; ++kk) {
      float ah[4], al[4], bh[4], bl[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ah[i] = ah_s[kk][ty + 16 * i];
        al[i] = al_s[kk][ty + 16 * i];
        bh[i] = bh_s[kk][tx + 16 * i];
        bl[i] = bl_s[kk][tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) mac(acc[i][j], ah[i], al[i], bh[j], bl[j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx + 16 * j;
      if (n < p.N) store_result(p.c, (b * p.M + m) * p.N + n, acc_final(acc[i][j]));
    }
  }
}

// Block-wide merge of Acc values; valid in thread 0.
__device__ Acc block_merge(Acc v) {
  __shared__ Acc part[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    Acc o{__shfl_down_sync(0xffffffffu, v.s, d), __shfl_down_sync(0xffffffffu, v.c, d)};
    v = acc_merge(v, o);
  }
  if (lane == 0) part[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? part[lane] : Acc{0.0f, 0.0f};
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      Acc o{__shfl_down_sync(0xffffffffu, v.s, d), __shfl_down_sync(0xffffffffu, v.c, d)};
      v = acc_merge(v, o);
    }
  }
  return v;
}

// grid = (splits, batch); block (s, b) folds k = s*T + t, stepping by splits*T.
__global__ void __launch_bounds__(kThreads)
dot_vec_kernel(DotProblem p, Acc* partials) {
  const int64_t b = blockIdx.y;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  Acc acc{0.0f, 0.0f};
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < p.K;
       k += step) {
    const ds2 x = load_ds(p.a, b * p.a.s_b + k * p.a.s_k);
    const ds2 y = load_ds(p.b, b * p.b.s_b + k * p.b.s_k);
    mac(acc, x.hi, x.lo, y.hi, y.lo);
  }
  acc = block_merge(acc);
  if (threadIdx.x == 0) {
    if (gridDim.x == 1)
      store_result(p.c, b, acc_final(acc));
    else
      partials[b * gridDim.x + blockIdx.x] = acc;
  }
}

__global__ void __launch_bounds__(kThreads)
dot_vec_finish_kernel(DotProblem p, const Acc* __restrict__ partials, int splits) {
  wait_previous_grid();  // the partials (a programmatic dependent launch)
  const int64_t b = blockIdx.x;
  Acc acc{0.0f, 0.0f};
  for (int i = threadIdx.x; i < splits; i += blockDim.x) acc = acc_merge(acc, partials[b * splits + i]);
  acc = block_merge(acc);
  if (threadIdx.x == 0) store_result(p.c, b, acc_final(acc));
}

}  // namespace

int dot_simt(const DotProblem& p, cudaStream_t s) {
  if (p.batch == 0 || p.M == 0 || p.N == 0) return ok();
  if (p.batch > 65535) return set_error(DS_INVALID_ARGUMENT, "dot_general: batch too large");
  const int64_t gy = (p.M + BM - 1) / BM;
  if (gy > 65535) return set_error(DS_INVALID_ARGUMENT, "dot_general: M too large for the CUDA-core path");
  dim3 grid(static_cast<unsigned>((p.N + BN - 1) / BN), static_cast<unsigned>(gy),
            static_cast<unsigned>(p.batch));
  ProfileScope prof("dot_simt", s);
  gemm_simt_kernel<<<grid, kThreads, 0, s>>>(p);
  return launch_status();
}

int dot_vec_splits(int64_t batch, int64_t K) {
  const int64_t by_len = (K + kThreads * 8 - 1) / (kThreads * 8);
  const int64_t by_fill = (static_cast<int64_t>(sm_count()) * 4 + batch - 1) / batch;
  int64_t g = by_len < by_fill ? by_len : by_fill;
  if (g < 1) g = 1;
  if (g > 1024) g = 1024;
  return static_cast<int>(g);
}

size_t dot_vec_workspace_bytes(int64_t batch, int64_t K) {
  const int g = dot_vec_splits(batch, K);
  return g > 1 ? static_cast<size_t>(batch) * g * sizeof(Acc) : 0;
}

int dot_batched_vec(const DotProblem& p, void* workspace, size_t workspace_bytes,
                    cudaStream_t s) {
  if (p.batch == 0) return ok();
  if (p.batch > 65535) return set_error(DS_INVALID_ARGUMENT, "dot_general: batch too large");
  const int g = dot_vec_splits(p.batch, p.K);
  const size_t need = dot_vec_workspace_bytes(p.batch, p.K);
  if (need > workspace_bytes || (need && !aligned(workspace, alignof(Acc))))
    return set_error(DS_INVALID_ARGUMENT, "dot_general: workspace too small");
  Acc* partials = static_cast<Acc*>(workspace);
  ProfileScope prof("dot_vec", s);
  dot_vec_kernel<<<dim3(g, static_cast<unsigned>(p.batch)), kThreads, 0, s>>>(p, partials);
  if (int st = launch_status()) return st;
  if (g > 1)
    DSB_CUDA_TRY(launch_dependent(dot_vec_finish_kernel, dim3(static_cast<unsigned>(p.batch)),
                                  dim3(kThreads), s, p, static_cast<const Acc*>(partials), g));
  return launch_status();
}

}  // namespace dsb
