// Event brackets around kernel launches (see profile.cu).
#pragma once

#include <cuda_runtime.h>

namespace dsb {

class ProfileScope {
 public:
  ProfileScope(const char* name, cudaStream_t s);
  ~ProfileScope();
  ProfileScope(const ProfileScope&) = delete;
  ProfileScope& operator=(const ProfileScope&) = delete;

 private:
  const char* name_;
  cudaStream_t stream_;
  cudaEvent_t start_ = nullptr;
};

}  // namespace dsb
