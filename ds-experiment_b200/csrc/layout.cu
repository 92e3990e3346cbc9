// Strided gather into a contiguous buffer: the copy that puts a dot_general
// operand whose batch, free or contracting dimensions do not nest into one
// stride each (e.g. free dimensions on both sides of a contracting one) into
// the [batch][rows][K] layout the products read.
#include "common.cuh"
#include "kernels.h"

namespace dsb {
namespace {

struct GatherDims {
  int nd;
  int64_t size[kGatherMaxDims];
  int64_t stride[kGatherMaxDims];
};

// dst[i] = src[offset(i)], i the row-major index over `size`, offset the sum
// of its digits times `stride` (elements).  Writes are coalesced; reads
// follow the source layout.
template <typename T>
__global__ void __launch_bounds__(256) gather_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                     int64_t n, GatherDims g) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t rem = i, off = 0;
#pragma unroll
    for (int d = kGatherMaxDims - 1; d >= 0; --d) {
      if (d < g.nd) {
        const int64_t q = rem / g.size[d];
        off += (rem - q * g.size[d]) * g.stride[d];
        rem = q;
      }
    }
    dst[i] = src[off];
  }
}

}  // namespace

int gather_strided(const void* src, void* dst, int elem_bytes, const int64_t* size,
                   const int64_t* stride, int nd, cudaStream_t s) {
  GatherDims g{};
  int64_t n = 1;
  for (int d = 0; d < nd; ++d) {
    if (size[d] == 1) continue;  // unit dimensions move nothing
    if (g.nd == kGatherMaxDims) return set_error(DS_INVALID_ARGUMENT, "gather: too many dimensions");
    g.size[g.nd] = size[d];
    g.stride[g.nd] = stride[d];
    ++g.nd;
    n *= size[d];
  }
  if (n == 0) return ok();
  const unsigned grid = grid_for(n, 256, 8);
  if (elem_bytes == 8) {
    gather_kernel<uint64_t><<<grid, 256, 0, s>>>(static_cast<const uint64_t*>(src),
                                                 static_cast<uint64_t*>(dst), n, g);
  } else if (elem_bytes == 4) {
    gather_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(src),
                                                 static_cast<uint32_t*>(dst), n, g);
  } else {
    return set_error(DS_INVALID_ARGUMENT, "gather: unsupported element size");
  }
  return launch_status();
}

}  // namespace dsb
