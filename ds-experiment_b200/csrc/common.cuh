// Shared plumbing of libds_b200: status codes, the per-thread error message,
// CUDA error checks, device properties and programmatic dependent launches.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "ds_b200.h"

namespace dsb {

// Sets the calling thread's last-error message and returns `code`.
int set_error(int code, const std::string& msg);
int ok();

// DS_INTERNAL with cudaGetErrorString, as the reference's CUDA handlers do
// (cpp/ds_fused_add_mul_to_f64_cuda.cu:118-121).
inline int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return ok();
  return set_error(DS_INTERNAL, cudaGetErrorString(err));
}

inline int launch_status() { return cuda_status(cudaGetLastError()); }

#define DSB_CUDA_TRY(expr)                          \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return cuda_status(_e);  \
  } while (0)

// Number of SMs of the current device (cached per device).
int sm_count();

// Grid for a grid-stride loop over `work` items with `threads` per block:
// enough blocks to fill every SM `per_sm` times, never more than needed.
inline unsigned grid_for(int64_t work, int threads, int per_sm) {
  const int64_t need = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  const int64_t g = need < cap ? need : cap;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

#ifdef __CUDACC__
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel on the stream finishes;
// it waits here, before reading anything that kernel wrote.  Without such a
// launch this returns at once.
__device__ __forceinline__ void wait_previous_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launch with programmatic stream serialization (see wait_previous_grid).
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, cudaStream_t s,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}
#endif

}  // namespace dsb
