// Exchange buffers shared between the processes of one node (one per GPU),
// mapped into every peer with CUDA IPC.  The owner allocates and zeroes the
// buffer and exports a handle; every other rank opens the handle, which maps
// the owner's memory into its address space with peer (NVLink) access
// enabled.  Plain cudaMalloc memory: no multicast object is involved, so a
// rank that exits leaves the others' memory untouched.
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace dsb {

size_t peer_handle_bytes() { return sizeof(cudaIpcMemHandle_t); }

int peer_alloc(size_t bytes, void** buf, void* handle) {
  if (buf == nullptr || handle == nullptr || bytes == 0)
    return set_error(DS_INVALID_ARGUMENT, "ds_exchange_alloc: null argument or zero size");
  void* p = nullptr;
  DSB_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e);
  }
  std::memcpy(handle, &h, sizeof h);
  *buf = p;
  return ok();
}

int peer_open(const void* handle, void** buf) {
  if (buf == nullptr || handle == nullptr)
    return set_error(DS_INVALID_ARGUMENT, "ds_exchange_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void* p = nullptr;
  DSB_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *buf = p;
  return ok();
}

int peer_close(void* buf) {
  if (buf == nullptr) return ok();
  DSB_CUDA_TRY(cudaIpcCloseMemHandle(buf));
  return ok();
}

int peer_free(void* buf) {
  if (buf == nullptr) return ok();
  DSB_CUDA_TRY(cudaFree(buf));
  return ok();
}

int peer_read_error(const void* buf, uint32_t* code) {
  if (buf == nullptr || code == nullptr)
    return set_error(DS_INVALID_ARGUMENT, "ds_exchange_error: null argument");
  DSB_CUDA_TRY(cudaMemcpy(code, static_cast<const unsigned char*>(buf) + kExchangeErrorOffset,
                          sizeof(uint32_t), cudaMemcpyDeviceToHost));
  return ok();
}

}  // namespace dsb
