// Tensor-core DS dot_general (int8 tcgen05, Ozaki scheme II).  Placeholder
// until the kernel lands: reports itself unsupported so dot_general takes
// the CUDA-core path.
#include "common.cuh"
#include "kernels.h"

namespace dsb {

bool dot_ozaki_supported(int64_t, int64_t, int64_t) { return false; }

size_t dot_ozaki_workspace_bytes(int64_t, int64_t, int64_t, int64_t) { return 0; }

int dot_ozaki(const DotProblem&, void*, size_t, cudaStream_t) {
  return set_error(DS_INTERNAL, "tensor-core dot_general not built");
}

}  // namespace dsb
