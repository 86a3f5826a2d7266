// Device status words: one int per device, zero while healthy. Kernels that time out in a bounded
// wait write a nonzero code (see common.cuh) with atomicCAS; the host polls and resets it.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAException.h>

#include <mutex>

#include "status.h"

namespace br {

static int* g_status[64] = {nullptr};
static std::mutex g_mu;

int* status_ptr(int device) {
  TORCH_CHECK(device >= 0 && device < 64, "bad device index");
  if (!g_status[device]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_status[device]) {
      c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
      int* p = nullptr;
      C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
      C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
      g_status[device] = p;
    }
  }
  return g_status[device];
}

int64_t read_status(int64_t device) {
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, status_ptr((int)device), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void reset_status(int64_t device) {
  C10_CUDA_CHECK(cudaMemset(status_ptr((int)device), 0, sizeof(int)));
}

}  // namespace br
