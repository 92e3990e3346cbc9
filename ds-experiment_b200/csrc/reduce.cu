// DS reduce: the reduce body of the DS pass (DsTransformPass.cpp:376-448,
// acc = ds_op(acc, elem) over (hi, lo) pairs) as CUDA kernels.
//
// Shapes are viewed as [outer, red, inner] (the reduced dimensions are
// contiguous).  Three kernels cover that:
//   - outer == 1, inner == 1 (a full reduction, e.g. jnp.sum of a vector):
//     every thread folds a grid-strided set of elements in index order (two
//     16-byte loads per step: f64 pairs, or hi/lo pairs), a warp shuffle tree
//     and a block tree combine threads, and block partials go to the caller's
//     workspace; a one-block kernel folds the partials with the same fixed
//     tree and applies init.  With one block the first kernel finishes alone.
//     For f64 input with an add/subtract body the per-thread fold is an
//     exact f64 two_sum of the inputs (see reduce_full_kernel).
//   - inner == 1, outer > 1: one block per row.
//   - inner > 1: one thread per (outer, inner) column, folding `red`
//     elements in order (coalesced across the inner index).
// Add and subtract bodies accumulate with ds_add (subtract: init - sum);
// multiply accumulates with ds_mul.  Every combine order is fixed by the
// shape, so results are deterministic.  HBM-bound for long inputs.
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "ds_arith.cuh"
#include "kernels.h"
#include "profile.h"

namespace dsb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;

__device__ __forceinline__ ds2 combine(bool is_mul, ds2 a, ds2 b) {
  return is_mul ? mul(a, b) : add(a, b);
}

__device__ __forceinline__ ds2 identity(bool is_mul) {
  return ds2{is_mul ? 1.0f : 0.0f, 0.0f};
}

__device__ __forceinline__ ds2 shfl_down(ds2 v, int d) {
  return ds2{__shfl_down_sync(0xffffffffu, v.hi, d), __shfl_down_sync(0xffffffffu, v.lo, d)};
}

// Block-wide fixed-order tree; the result is valid in thread 0.
__device__ ds2 block_combine(bool is_mul, ds2 v) {
  __shared__ ds2 warp_part[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = combine(is_mul, v, shfl_down(v, d));
  if (lane == 0) warp_part[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kWarps ? warp_part[lane] : identity(is_mul);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = combine(is_mul, v, shfl_down(v, d));
  }
  return v;
}

// Final step shared by every kernel: fold init in once, then write.
__device__ __forceinline__ ds2 finish(int body, ds2 init, ds2 total) {
  return body == 2 ? mul(init, total) : (body == 1 ? sub(init, total) : add(init, total));
}

struct Src {
  const double* f64;  // f64 input (split on load), or
  const float* hi;    // SoA DS input (packed: hi = the [..., 2] array, lo unused)
  const float* lo;
  bool vec;           // 16-byte aligned pair loads allowed
  bool packed;        // packed DS input: element i at hi[2i], hi[2i + 1]
  __device__ __forceinline__ ds2 at(int64_t i) const {
    if (f64) return from_f64(f64[i]);
    return packed ? ds2{hi[2 * i], hi[2 * i + 1]} : ds2{hi[i], lo[i]};
  }
  __device__ __forceinline__ void pair(int64_t p, ds2& x0, ds2& x1) const {
    if (f64) {
      const double2 v = __ldcs(reinterpret_cast<const double2*>(f64) + p);
      x0 = from_f64(v.x);
      x1 = from_f64(v.y);
    } else if (packed) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(hi) + p);
      x0 = ds2{v.x, v.y};
      x1 = ds2{v.z, v.w};
    } else {
      const float2 h = __ldcs(reinterpret_cast<const float2*>(hi) + p);
      const float2 l = __ldcs(reinterpret_cast<const float2*>(lo) + p);
      x0 = ds2{h.x, l.x};
      x1 = ds2{h.y, l.y};
    }
  }
};

struct Dst {
  double* f64;  // f64 output, or
  float* hi;    // SoA DS output
  float* lo;
  __device__ __forceinline__ void put(int64_t i, ds2 v) const {
    if (f64) {
      f64[i] = to_f64(v);
    } else {
      hi[i] = v.hi;
      lo[i] = v.lo;
    }
  }
};

__device__ __forceinline__ ds2 load_init(const double* init_f64, const float* init_hi,
                                         const float* init_lo) {
  return init_f64 ? from_f64(*init_f64) : ds2{*init_hi, *init_lo};
}

// Knuth two_sum in f64: s + c += x with the rounding error of s + x kept in c.
__device__ __forceinline__ void two_sum_acc(double& s, double& c, double x) {
  const double t = __dadd_rn(s, x);
  const double bp = __dsub_rn(t, s);
  c = __dadd_rn(c, __dadd_rn(__dsub_rn(s, __dsub_rn(t, bp)), __dsub_rn(x, bp)));
  s = t;
}

// Full reduction, stage 1.
//
// f64 input with an add/subtract body: every thread sums its elements
// exactly in f64 (two_sum, the rounding errors carried in a second f64), and
// its partial enters the DS trees as the DS split of that sum.  This adds the
// f64 inputs themselves -- splitting each into (hi, lo) first would only add
// a rounding per element -- with no f64->f32 conversion per element.  Other
// inputs and the multiply body fold DS pairs.
__global__ void __launch_bounds__(kThreads)
reduce_full_kernel(Src src, int64_t n, int body, ds2* partials, Dst dst,
                   const double* init_f64, const float* init_hi, const float* init_lo,
                   bool always_partials = false) {
  wait_previous_grid();  // launched as a programmatic dependent: the producer's writes
  const bool is_mul = body == 2;
  ds2 acc = identity(is_mul);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (src.f64 && !is_mul && src.vec) {
    double s0 = 0.0, c0 = 0.0, s1 = 0.0, c1 = 0.0;
    const int64_t npairs = n >> 1;
    const double2* p2 = reinterpret_cast<const double2*>(src.f64);
    for (int64_t base = tid; base < npairs; base += stride * kUnroll) {
      double2 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t p = base + u * stride;
        v[u] = p < npairs ? __ldcs(p2 + p) : make_double2(0.0, 0.0);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        two_sum_acc(s0, c0, v[u].x);
        two_sum_acc(s1, c1, v[u].y);
      }
    }
    if ((n & 1) && tid == 0) two_sum_acc(s0, c0, src.f64[n - 1]);
    two_sum_acc(s0, c0, s1);
    acc = from_f64(__dadd_rn(s0, __dadd_rn(c0, c1)));
  } else if (src.vec) {
    const int64_t npairs = n >> 1;
    for (int64_t base = tid; base < npairs; base += stride * kUnroll) {
      ds2 x0[kUnroll], x1[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t p = base + u * stride;
        if (p < npairs) src.pair(p, x0[u], x1[u]);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t p = base + u * stride;
        if (p < npairs) {
          acc = combine(is_mul, acc, x0[u]);
          acc = combine(is_mul, acc, x1[u]);
        }
      }
    }
    if ((n & 1) && tid == 0) acc = combine(is_mul, acc, src.at(n - 1));
  } else {
    for (int64_t i = tid; i < n; i += stride) acc = combine(is_mul, acc, src.at(i));
  }
  acc = block_combine(is_mul, acc);
  if (threadIdx.x == 0) {
    if (gridDim.x == 1 && !always_partials) {
      // An empty reduction returns init unchanged (bits included).
      const ds2 init = load_init(init_f64, init_hi, init_lo);
      dst.put(0, n == 0 ? init : finish(body, init, acc));
    } else {
      partials[blockIdx.x] = acc;
    }
  }
}

// Full reduction of long aligned f64 input (add / subtract body), stage 1,
// as a bulk-copy stream: each block owns every G-th chunk of kBulkChunk
// values and keeps kBulkStages chunks in flight with cp.async.bulk into
// shared memory (one mbarrier per stage), so the bytes in flight do not
// depend on registers or occupancy.  The threads fold the values of a chunk
// exactly in f64 (two_sum, as reduce_full_kernel) and the block writes one
// DS partial.  Block 0 also folds the last n mod kBulkChunk values.  Every
// wait is bounded; a block whose wait runs out stops issuing, waits (bounded)
// for its copies in flight and writes a NaN partial, so the result is NaN.
// One block per SM with two 64 KB chunks in flight: at 2^26 values 6.32 TB/s,
// against 6.0-6.1 with two blocks of three 32 KB chunks each and 5.7 with
// six 32 KB chunks in one block (fewer, larger copies win).
constexpr int kBulkChunk = 8192;  // values per chunk (64 KB)
constexpr int kBulkStages = 2;
constexpr int kBulkBlocksPerSm = 1;
constexpr long long kBulkTimeoutCycles = 2000000000LL;  // ~1 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool bulk_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kBulkTimeoutCycles) return false;
  }
}

__device__ __forceinline__ void bulk_issue(double* dst, const double* src, uint32_t bytes,
                                           uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__global__ void __launch_bounds__(kThreads)
reduce_bulk_kernel(const double* __restrict__ x, int64_t n, ds2* __restrict__ partials) {
  extern __shared__ __align__(128) unsigned char smem[];
  double* buf = reinterpret_cast<double*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBulkStages * kBulkChunk * sizeof(double));
  const int64_t nchunks = n / kBulkChunk;
  const int64_t G = gridDim.x;
  const int64_t mine = nchunks > blockIdx.x ? (nchunks - blockIdx.x + G - 1) / G : 0;
  constexpr uint32_t kBytes = kBulkChunk * sizeof(double);
  if (threadIdx.x == 0) {
    for (int st = 0; st < kBulkStages; ++st)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[st])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int64_t i = 0; i < kBulkStages && i < mine; ++i)
      bulk_issue(buf + i * kBulkChunk, x + (blockIdx.x + i * G) * kBulkChunk, kBytes, &full[i]);
  }
  __syncthreads();
  double s0 = 0.0, c0 = 0.0, s1 = 0.0, c1 = 0.0;
  bool failed = false;
  int64_t consumed = 0;
  for (int64_t i = 0; i < mine; ++i) {
    const int st = static_cast<int>(i % kBulkStages);
    const uint32_t parity = static_cast<uint32_t>((i / kBulkStages) & 1);
    const bool arrived = bulk_wait(&full[st], parity);
    if (__syncthreads_or(!arrived)) {
      failed = true;
      break;
    }
    const double2* p = reinterpret_cast<const double2*>(buf + st * kBulkChunk) + threadIdx.x;
#pragma unroll
    for (int u = 0; u < kBulkChunk / 2 / kThreads; ++u) {
      const double2 v = p[u * kThreads];
      two_sum_acc(s0, c0, v.x);
      two_sum_acc(s1, c1, v.y);
    }
    consumed = i + 1;
    __syncthreads();  // every read of this stage is done before it is refilled
    if (threadIdx.x == 0 && i + kBulkStages < mine) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bulk_issue(buf + st * kBulkChunk, x + (blockIdx.x + (i + kBulkStages) * G) * kBulkChunk,
                 kBytes, &full[st]);
    }
  }
  if (failed && threadIdx.x == 0) {
    // wait (bounded) for the copies still in flight before the block exits
    const int64_t issued = mine < consumed + kBulkStages ? mine : consumed + kBulkStages;
    for (int64_t i = consumed; i < issued; ++i)
      bulk_wait(&full[i % kBulkStages], static_cast<uint32_t>((i / kBulkStages) & 1));
  }
  if (blockIdx.x == 0) {
    for (int64_t i = nchunks * kBulkChunk + threadIdx.x; i < n; i += kThreads)
      two_sum_acc(s0, c0, __ldcs(x + i));
  }
  two_sum_acc(s0, c0, s1);
  ds2 acc = from_f64(__dadd_rn(s0, __dadd_rn(c0, c1)));
  acc = block_combine(false, acc);
  if (threadIdx.x == 0) {
    const float nan = __int_as_float(0x7fffffff);
    partials[blockIdx.x] = failed ? ds2{nan, nan} : acc;
  }
}

// Full reduction, stage 2: one block folds the G partials.  Launched as a
// programmatic dependent of stage 1, so its launch overlaps stage 1's tail.
__global__ void __launch_bounds__(kThreads)
reduce_partials_kernel(const ds2* __restrict__ partials, int g, int body, Dst dst,
                       const double* init_f64, const float* init_hi, const float* init_lo) {
  wait_previous_grid();  // stage 1's partials
  const bool is_mul = body == 2;
  ds2 acc = identity(is_mul);
  for (int i = threadIdx.x; i < g; i += blockDim.x) acc = combine(is_mul, acc, partials[i]);
  acc = block_combine(is_mul, acc);
  if (threadIdx.x == 0) dst.put(0, finish(body, load_init(init_f64, init_hi, init_lo), acc));
}

// inner == 1, outer > 1, rows of at least kRowsBlockMin values: one block per row.
__global__ void __launch_bounds__(kThreads)
reduce_rows_kernel(Src src, int64_t outer, int64_t red, int body, Dst dst,
                   const double* init_f64, const float* init_hi, const float* init_lo) {
  const bool is_mul = body == 2;
  const ds2 init = load_init(init_f64, init_hi, init_lo);
  for (int64_t row = blockIdx.x; row < outer; row += gridDim.x) {
    ds2 acc = identity(is_mul);
    const int64_t off = row * red;
    for (int64_t r = threadIdx.x; r < red; r += blockDim.x)
      acc = combine(is_mul, acc, src.at(off + r));
    acc = block_combine(is_mul, acc);
    if (threadIdx.x == 0) dst.put(row, red == 0 ? init : finish(body, init, acc));
    __syncthreads();
  }
}

// inner == 1, rows shorter than kRowsBlockMin: groups of `lanes` lanes (a
// power of two up to 32, about eight values per lane) fold one row each.
// The row loop advances a warp at a time, so every lane reaches every
// shuffle; a group past the last row folds nothing and writes nothing.
constexpr int64_t kRowsBlockMin = 2048;

int rows_lanes(int64_t red) {
  int lanes = 1;
  while (lanes < 32 && static_cast<int64_t>(lanes) * 8 < red) lanes <<= 1;
  return lanes;
}

__global__ void __launch_bounds__(kThreads)
reduce_rows_groups_kernel(Src src, int64_t outer, int64_t red, int lanes, int body, Dst dst,
                          const double* init_f64, const float* init_hi, const float* init_lo) {
  const bool is_mul = body == 2;
  const ds2 init = load_init(init_f64, init_hi, init_lo);
  const int lane = threadIdx.x & 31, sub = lane % lanes, per_warp = 32 / lanes;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = wid * per_warp; base < outer; base += nw * per_warp) {
    const int64_t row = base + lane / lanes;
    ds2 acc = identity(is_mul);
    if (row < outer) {
      const int64_t off = row * red;
      for (int64_t r = sub; r < red; r += lanes) acc = combine(is_mul, acc, src.at(off + r));
    }
    for (int o = lanes >> 1; o > 0; o >>= 1) {
      const ds2 t{__shfl_xor_sync(0xffffffffu, acc.hi, o), __shfl_xor_sync(0xffffffffu, acc.lo, o)};
      acc = combine(is_mul, acc, t);
    }
    if (sub == 0 && row < outer) dst.put(row, red == 0 ? init : finish(body, init, acc));
  }
}

// inner > 1: one thread per (outer, inner) column.
__global__ void __launch_bounds__(kThreads)
reduce_cols_kernel(Src src, int64_t outer, int64_t red, int64_t inner, int body, Dst dst,
                   const double* init_f64, const float* init_hi, const float* init_lo) {
  const bool is_mul = body == 2;
  const ds2 init = load_init(init_f64, init_hi, init_lo);
  const int64_t cols = outer * inner;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < cols;
       c += stride) {
    const int64_t o = c / inner, j = c - o * inner;
    const int64_t off = o * red * inner + j;
    ds2 acc = identity(is_mul);
    for (int64_t r = 0; r < red; ++r) acc = combine(is_mul, acc, src.at(off + r * inner));
    dst.put(c, red == 0 ? init : finish(body, init, acc));
  }
}

// inner > 1 with too few columns to fill the GPU one thread each: a block
// owns 32 adjacent columns, its 8 warps split the reduced dimension (warp w
// folds positions w, w + 8, ...; loads stay coalesced along the columns),
// and the 8 partials of a column are folded in warp order.
__global__ void __launch_bounds__(kThreads)
reduce_cols_tile_kernel(Src src, int64_t outer, int64_t red, int64_t inner, int body, Dst dst,
                        const double* init_f64, const float* init_hi, const float* init_lo) {
  wait_previous_grid();  // as the sliced path's second pass: the slices' partials
  __shared__ ds2 part[kThreads / 32][32];
  const bool is_mul = body == 2;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t cols = outer * inner;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * 32 + tx;
  ds2 acc = identity(is_mul);
  if (c < cols) {
    const int64_t o = c / inner, j = c - o * inner;
    const int64_t off = o * red * inner + j;
    for (int64_t r = ty; r < red; r += kThreads / 32)
      acc = combine(is_mul, acc, src.at(off + r * inner));
  }
  part[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < cols) {
    ds2 t = part[0][tx];
    for (int w = 1; w < kThreads / 32; ++w) t = combine(is_mul, t, part[w][tx]);
    const ds2 init = load_init(init_f64, init_hi, init_lo);
    dst.put(c, red == 0 ? init : finish(body, init, t));
  }
}

// The tile kernel's first stage when a few columns have long reductions:
// grid (tiles, slices); block (x, s) folds rows [s * chunk, (s + 1) * chunk)
// of its 32 columns (8 warps, as above) and writes the slice's DS partial
// per column to partials[s * cols + c], without init.
__global__ void __launch_bounds__(kThreads)
reduce_cols_split_kernel(Src src, int64_t outer, int64_t red, int64_t inner, int64_t chunk,
                         int body, ds2* __restrict__ partials) {
  __shared__ ds2 part[kThreads / 32][32];
  const bool is_mul = body == 2;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t cols = outer * inner;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * 32 + tx;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * chunk;
  const int64_t r1 = r0 + chunk < red ? r0 + chunk : red;
  ds2 acc = identity(is_mul);
  if (c < cols) {
    const int64_t o = c / inner, j = c - o * inner;
    const int64_t off = o * red * inner + j;
    for (int64_t r = r0 + ty; r < r1; r += kThreads / 32)
      acc = combine(is_mul, acc, src.at(off + r * inner));
  }
  part[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < cols) {
    ds2 t = part[0][tx];
    for (int w = 1; w < kThreads / 32; ++w) t = combine(is_mul, t, part[w][tx]);
    partials[static_cast<int64_t>(blockIdx.y) * cols + c] = t;
  }
}

// Slices of the reduced dimension for the split column reduction: about
// kSliceBlocks blocks (a B200 holds 8 per SM, 1184), at least 1024 rows a
// slice, at most 512 slices; 1 (no split) when the columns alone make half
// that many blocks or the rows are short.  A function of the shape alone,
// so the summation order (and the bits) do not depend on the device.
constexpr int64_t kSliceBlocks = 1024;

int64_t cols_slices(int64_t outer, int64_t red, int64_t inner) {
  if (inner <= 1) return 1;
  const int64_t tiles = (outer * inner + 31) / 32;
  const int64_t want = kSliceBlocks;
  if (tiles >= want / 2 || red < 4096) return 1;
  int64_t sl = (want + tiles - 1) / tiles;
  if (sl > red / 1024) sl = red / 1024;
  if (sl > 512) sl = 512;
  return sl < 2 ? 1 : sl;
}

}  // namespace

int reduce_full_blocks(int64_t n) {
  return static_cast<int>(grid_for((n + 2 * kUnroll - 1) / (2 * kUnroll), kThreads, 8));
}

size_t reduce_workspace_bytes(int64_t outer, int64_t red, int64_t inner) {
  if (inner > 1) {
    const int64_t sl = cols_slices(outer, red, inner);
    return sl > 1 ? static_cast<size_t>(sl * outer * inner) * sizeof(ds2) : 0;
  }
  if (outer != 1 || inner != 1) return 0;
  const int g = reduce_full_blocks(red);
  return g > 1 ? static_cast<size_t>(g) * sizeof(ds2) : 0;
}

namespace {

// Long aligned f64 input with an add/subtract body takes the bulk-copy
// kernel; 16 B alignment is what cp.async.bulk needs.
constexpr int64_t kBulkMinElements = int64_t(1) << 20;

bool use_bulk(const Src& src, int64_t n, int body) {
  return src.f64 != nullptr && src.vec && body != 2 && n >= kBulkMinElements;
}

int bulk_blocks() { return sm_count() * kBulkBlocksPerSm; }

size_t bulk_smem_bytes() {
  return static_cast<size_t>(kBulkStages) * kBulkChunk * sizeof(double) +
         kBulkStages * sizeof(uint64_t);
}

// Stage 1 of a full reduction into `partials`; returns the number of
// partials, or -1 after a launch error (the error is set).  With one block
// and !always_partials the old kernel writes the result directly.
int full_stage1(const Src& src, int64_t n, int body, ds2* partials, Dst dst,
                const double* init_f64, const float* init_hi, const float* init_lo,
                bool always_partials, cudaStream_t s) {
  if (use_bulk(src, n, body)) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
      attr_err = cudaFuncSetAttribute(reduce_bulk_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(bulk_smem_bytes()));
    });
    if (attr_err != cudaSuccess) {
      cuda_status(attr_err);
      return -1;
    }
    const int g = bulk_blocks();
    reduce_bulk_kernel<<<g, kThreads, bulk_smem_bytes(), s>>>(src.f64, n, partials);
    return launch_status() == DS_OK ? g : -1;
  }
  const int g = n == 0 ? 1 : reduce_full_blocks(n);
  if (cuda_status(launch_dependent(reduce_full_kernel, dim3(g), dim3(kThreads), s, src, n, body,
                                   partials, dst, init_f64, init_hi, init_lo,
                                   always_partials)) != DS_OK)
    return -1;
  return launch_status() == DS_OK ? g : -1;
}

}  // namespace

int reduce_launch(const ReduceArgs& a, cudaStream_t s) {
  Src src{a.in_f64, a.in_packed ? a.in_packed : a.in_hi, a.in_lo, false, a.in_packed != nullptr};
  src.vec = a.in_f64      ? aligned(a.in_f64, 16)
            : src.packed ? aligned(a.in_packed, 16)
                         : (aligned(a.in_hi, 8) && aligned(a.in_lo, 8));
  Dst dst{a.out_f64, a.out_hi, a.out_lo};
  const int64_t outer = a.outer, red = a.red, inner = a.inner;
  if (outer * inner == 0) return ok();
  if (outer == 1 && inner == 1) {
    const int g = red == 0 ? 1 : reduce_full_blocks(red);
    const size_t need = g > 1 ? static_cast<size_t>(g) * sizeof(ds2) : 0;
    if (need > a.workspace_bytes || (need && !aligned(a.workspace, alignof(ds2)))) {
      return set_error(DS_INVALID_ARGUMENT,
                       "ds_reduce: workspace too small (need " + std::to_string(need) +
                           " bytes, 8-byte aligned)");
    }
    ds2* partials = static_cast<ds2*>(a.workspace);
    ProfileScope prof("reduce", s);
    const int used = full_stage1(src, red, a.body, partials, dst, a.init_f64, a.init_hi,
                                 a.init_lo, false, s);
    if (used < 0) return DS_INTERNAL;
    if (used > 1) {
      DSB_CUDA_TRY(launch_dependent(reduce_partials_kernel, dim3(1), dim3(kThreads), s,
                                    static_cast<const ds2*>(partials), used, a.body, dst,
                                    a.init_f64, a.init_hi, a.init_lo));
    }
    return launch_status();
  }
  if (inner == 1) {
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    if (red < kRowsBlockMin) {
      const int lanes = rows_lanes(red);
      const int64_t need = (outer + kThreads / lanes - 1) / (kThreads / lanes);
      const unsigned g = static_cast<unsigned>(need < cap ? need : cap);
      reduce_rows_groups_kernel<<<g, kThreads, 0, s>>>(src, outer, red, lanes, a.body, dst,
                                                       a.init_f64, a.init_hi, a.init_lo);
      return launch_status();
    }
    const unsigned g = static_cast<unsigned>(outer < cap ? outer : cap);
    reduce_rows_kernel<<<g, kThreads, 0, s>>>(src, outer, red, a.body, dst, a.init_f64,
                                              a.init_hi, a.init_lo);
    return launch_status();
  }
  if (outer * inner < static_cast<int64_t>(sm_count()) * kThreads * 8) {
    const int64_t tiles = (outer * inner + 31) / 32;
    const int64_t sl = cols_slices(outer, red, inner);
    const size_t need = static_cast<size_t>(sl * outer * inner) * sizeof(ds2);
    if (sl > 1 && a.workspace && a.workspace_bytes >= need && aligned(a.workspace, alignof(ds2))) {
      // long reductions over few columns: slices in parallel, then the
      // slices' partials folded in slice order with init (a workspace too
      // small for them keeps the one-stage kernel below)
      ds2* partials = static_cast<ds2*>(a.workspace);
      const int64_t chunk = (red + sl - 1) / sl;
      reduce_cols_split_kernel<<<dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(sl)),
                                 kThreads, 0, s>>>(src, outer, red, inner, chunk, a.body,
                                                   partials);
      if (int st = launch_status()) return st;
      Src ps{nullptr, reinterpret_cast<const float*>(partials), nullptr, false, true};
      DSB_CUDA_TRY(launch_dependent(reduce_cols_tile_kernel,
                                    dim3(static_cast<unsigned>(tiles)), dim3(kThreads), s, ps,
                                    int64_t{1}, sl, outer * inner, a.body, dst, a.init_f64,
                                    a.init_hi, a.init_lo));
      return launch_status();
    }
    reduce_cols_tile_kernel<<<static_cast<unsigned>(tiles), kThreads, 0, s>>>(
        src, outer, red, inner, a.body, dst, a.init_f64, a.init_hi, a.init_lo);
    return launch_status();
  }
  reduce_cols_kernel<<<grid_for(outer * inner, kThreads, 8), kThreads, 0, s>>>(
      src, outer, red, inner, a.body, dst, a.init_f64, a.init_hi, a.init_lo);
  return launch_status();
}

// ---- allocation-free variant ------------------------------------------------
//
// For callers that cannot allocate device memory (see ds_reduce_f64_noalloc
// in ds_b200.h), the partials that ds_reduce_f64 keeps in caller workspace
// live in this file-scope device array instead: the block partials of a full
// reduction (at most 8 per SM), or the slice partials of a reduction over a
// leading dimension with few columns (slices * columns, below
// 32 * (kSliceBlocks + 512) = 49152 by cols_slices).  Every GPU that loads
// the library holds it (384 KiB) until the process exits.  Host code cannot
// use the symbol itself as a pointer (on the host it names a stand-in, not
// device memory), so its device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, and passed to the kernels.
// All calls share the array: the first stage overwrites every slot that the
// second reads, so nothing needs clearing between calls, but two calls whose
// kernels overlap on the GPU (different streams, no ordering) race on it.

constexpr int kStaticPartials = 49152;
static __device__ __align__(256) ds2 g_static_partials[kStaticPartials];

namespace {

int static_partials_address(ds2** out) {
  static std::mutex mu;
  static std::vector<ds2*> by_device;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(by_device.size())) by_device.resize(dev + 1, nullptr);
  if (by_device[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_partials);
    if (e != cudaSuccess) return cuda_status(e);
    by_device[dev] = static_cast<ds2*>(p);
  }
  *out = by_device[dev];
  return ok();
}

}  // namespace

int reduce_launch_noalloc(ReduceArgs a, cudaStream_t s) {
  const size_t need = reduce_workspace_bytes(a.outer, a.red, a.inner);
  if (need > sizeof(g_static_partials)) {
    return set_error(DS_INVALID_ARGUMENT,
                     "ds_reduce_f64_noalloc: needs " + std::to_string(need / sizeof(ds2)) +
                         " partials, more than its static maximum of " +
                         std::to_string(kStaticPartials));
  }
  if (need > 0) {
    ds2* partials = nullptr;
    if (int st = static_partials_address(&partials)) return st;
    a.workspace = partials;
    a.workspace_bytes = need;
  }
  return reduce_launch(a, s);
}

// ---- sharded full reduction: the totals exchanged over peer memory ----------
//
// Every rank (one process per GPU) reduces its own shard to a DS total, and
// one kernel then publishes that total to every rank's exchange buffer with
// plain stores through peer (NVLink P2P) mappings, waits -- bounded -- until
// the totals of all ranks have arrived in its own buffer, and folds them in
// rank order, so every rank writes the same bits.  No collective library and
// no host round trip sit between the local reduce and the result.
//
// Exchange buffer of one rank (kExchangeBytes, zeroed at allocation):
//   records[2][kExchangeMaxRanks] of 32 bytes at offset (parity * 8 + r) * 32:
//     f32 hi, f32 lo, i64 n (elements of rank r's shard), u64 epoch, u64 pad
//   u32 error word at kExchangeErrorOffset (sticky; 1 = a wait timed out).
// Call number `epoch` (1, 2, ... -- the same sequence on every rank) uses the
// records of parity epoch & 1.  A rank reaches call e + 2, and overwrites
// those records again, only after every other rank has published call e + 1,
// which each does only after it finished reading call e: two parities keep a
// fast rank from overwriting records a slow one still has to read.
// The writer stores hi, lo, n, then a system-scope fence, then the epoch with
// a release store; the reader acquires the epoch before reading the rest.

namespace {

struct __align__(16) ExchangeRecord {
  float hi, lo;
  long long n;
  unsigned long long epoch;
  unsigned long long pad;
};
static_assert(sizeof(ExchangeRecord) == 32, "exchange record layout");
static_assert(2 * kExchangeMaxRanks * sizeof(ExchangeRecord) <= kExchangeErrorOffset,
              "exchange records overlap the error word");

struct ExchangePeers {
  unsigned char* buf[kExchangeMaxRanks];
};

__device__ __forceinline__ ExchangeRecord* exchange_record(unsigned char* buf, int parity,
                                                           int r) {
  return reinterpret_cast<ExchangeRecord*>(buf) + parity * kExchangeMaxRanks + r;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Stage 2 of a sharded full reduction (one block): fold this rank's block
// partials (the same fixed tree as reduce_partials_kernel), exchange the
// totals, fold the non-empty ranks' totals in rank order and apply init.
// On a timed-out wait the result is NaN and the error word is set.
__global__ void __launch_bounds__(kThreads)
reduce_exchange_kernel(const ds2* __restrict__ partials, int g, long long n_local, int body,
                       Dst dst, const double* init_f64, ExchangePeers peers, int world, int rank,
                       unsigned long long epoch, long long timeout_ns) {
  __shared__ ds2 totals[kExchangeMaxRanks];
  __shared__ long long counts[kExchangeMaxRanks];
  __shared__ int failed;
  const bool is_mul = body == 2;
  ds2 acc = identity(is_mul);
  for (int i = threadIdx.x; i < g; i += blockDim.x) acc = combine(is_mul, acc, partials[i]);
  acc = block_combine(is_mul, acc);
  const int parity = static_cast<int>(epoch & 1ull);
  if (threadIdx.x == 0) {
    failed = 0;
    for (int r = 0; r < world; ++r) {
      volatile ExchangeRecord* rec = exchange_record(peers.buf[r], parity, rank);
      rec->hi = acc.hi;
      rec->lo = acc.lo;
      rec->n = n_local;
    }
    __threadfence_system();
    for (int r = 0; r < world; ++r)
      store_release_sys(&exchange_record(peers.buf[r], parity, rank)->epoch, epoch);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    ExchangeRecord* rec = exchange_record(peers.buf[rank], parity, threadIdx.x);
    const unsigned long long t0 = global_ns();
    bool arrived = true;
    while (load_acquire_sys(&rec->epoch) != epoch) {
      if (static_cast<long long>(global_ns() - t0) > timeout_ns) {
        arrived = false;
        break;
      }
      __nanosleep(128);
    }
    if (arrived) {
      const volatile ExchangeRecord* v = rec;
      totals[threadIdx.x] = ds2{v->hi, v->lo};
      counts[threadIdx.x] = v->n;
    } else {
      failed = 1;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (failed) {
      atomicOr(reinterpret_cast<unsigned*>(peers.buf[rank] + kExchangeErrorOffset), 1u);
      const float nan = __int_as_float(0x7fffffff);
      dst.put(0, ds2{nan, nan});
      return;
    }
    const ds2 init = load_init(init_f64, nullptr, nullptr);
    bool any = false;
    ds2 total = identity(is_mul);
    for (int r = 0; r < world; ++r) {
      if (counts[r] == 0) continue;
      total = any ? combine(is_mul, total, totals[r]) : totals[r];
      any = true;
    }
    dst.put(0, any ? finish(body, init, total) : init);
  }
}

}  // namespace

size_t reduce_sharded_workspace_bytes(int64_t n) {
  return static_cast<size_t>(n > 0 ? reduce_full_blocks(n) : 1) * sizeof(ds2);
}

int reduce_sharded_launch(const ShardedReduceArgs& a, cudaStream_t s) {
  if (a.world < 1 || a.world > kExchangeMaxRanks || a.rank < 0 || a.rank >= a.world)
    return set_error(DS_INVALID_ARGUMENT, "ds_reduce_f64_sharded: invalid rank/world");
  const int g = a.n > 0 ? reduce_full_blocks(a.n) : 1;
  const size_t need = static_cast<size_t>(g) * sizeof(ds2);
  if (need > a.workspace_bytes || !aligned(a.workspace, alignof(ds2)))
    return set_error(DS_INVALID_ARGUMENT,
                     "ds_reduce_f64_sharded: workspace too small (need " +
                         std::to_string(need) + " bytes, 8-byte aligned)");
  ExchangePeers peers{};
  for (int r = 0; r < a.world; ++r) {
    if (a.buffers[r] == nullptr || !aligned(a.buffers[r], 16))
      return set_error(DS_INVALID_ARGUMENT,
                       "ds_reduce_f64_sharded: exchange buffers must be 16-byte aligned");
    peers.buf[r] = static_cast<unsigned char*>(a.buffers[r]);
  }
  Src src{a.in, nullptr, nullptr, aligned(a.in, 16), false};
  Dst dst{a.out, nullptr, nullptr};
  ds2* partials = static_cast<ds2*>(a.workspace);
  ProfileScope prof("reduce", s);
  const int used = full_stage1(src, a.n, a.body, partials, dst, nullptr, nullptr, nullptr, true, s);
  if (used < 0) return DS_INTERNAL;
  reduce_exchange_kernel<<<1, kThreads, 0, s>>>(partials, used, a.n, a.body, dst, a.init, peers,
                                                a.world, a.rank, a.epoch, a.timeout_ns);
  return launch_status();
}

}  // namespace dsb
