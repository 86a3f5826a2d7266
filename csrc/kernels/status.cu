// Device status words: one int per device, zero while healthy. Kernels that time out in a bounded
// wait write a nonzero code (see common.cuh) with atomicCAS; the host polls and resets it.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAStream.h>

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

// Queues a copy of the status word (and of a device skip word, if given) into out (int32, pinned host
// memory, >= 2 entries) on the current stream, so the host can read them later without a device sync.
void status_snapshot(torch::Tensor& out, c10::optional<torch::Tensor> skip) {
  TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() >= 2 && !out.is_cuda() && out.is_pinned(),
              "status_snapshot: pinned int32 host tensor with 2 entries");
  const int dev = skip.has_value() && skip->defined() ? skip->device().index() : c10::cuda::current_device();
  c10::cuda::CUDAGuard g((c10::DeviceIndex)dev);
  auto st = c10::cuda::getCurrentCUDAStream();
  int* o = out.data_ptr<int>();
  C10_CUDA_CHECK(cudaMemcpyAsync(o, status_ptr(dev), sizeof(int), cudaMemcpyDeviceToHost, st));
  if (skip.has_value() && skip->defined())
    C10_CUDA_CHECK(cudaMemcpyAsync(o + 1, skip->data_ptr<int>(), sizeof(int), cudaMemcpyDeviceToHost, st));
}

}  // namespace br
