// Allocation-free variant of the Muon momentum + normalisation kernels (see muon_noalloc.h).
//
// Same math as muon_momentum_kernel / muon_normalize_kernel in optim.cu, for matrices stored back to
// back instead of a pointer list, with the per-matrix sum of squares kept in a file-scope __device__
// array instead of a caller-allocated buffer. Nothing here calls cudaMalloc, cudaFree or any library
// routine that allocates.
#include "muon_noalloc.h"

#include <mutex>

namespace {

// Per-matrix sum of squares of the Nesterov gradient (the only scratch the step needs).
static __device__ __align__(256) float g_muon_ss[BR_MUON_NOALLOC_MAX_MATRICES];

__global__ void noalloc_clear_kernel(float* ss, int S) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < S; i += gridDim.x * blockDim.x) ss[i] = 0.f;
}

// grid (chunks, S): momentum update in place and sum((g')^2) per matrix into ss[s]
__global__ void noalloc_momentum_kernel(const float* __restrict__ grad, float* __restrict__ mom, int64_t n, float mu,
                                        float* __restrict__ ss) {
  const int s = blockIdx.y;
  const float* g = grad + (int64_t)s * n;
  float* m = mom + (int64_t)s * n;
  float acc = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i];
    const float mi = mu * m[i] + (1.f - mu) * gi;
    m[i] = mi;
    const float gp = (1.f - mu) * gi + mu * mi;
    acc += gp * gp;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(ss + s, acc);
}

__global__ void noalloc_normalize_kernel(const float* __restrict__ grad, const float* __restrict__ mom, int64_t n,
                                         float mu, const float* __restrict__ ss, __nv_bfloat16* __restrict__ x) {
  const int s = blockIdx.y;
  const float* g = grad + (int64_t)s * n;
  const float* m = mom + (int64_t)s * n;
  __nv_bfloat16* xo = x + (int64_t)s * n;
  const float inv = 1.f / (sqrtf(ss[s]) * 1.02f + 1e-6f);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    xo[i] = __float2bfloat16(((1.f - mu) * g[i] + mu * m[i]) * inv);
}

// Device address of g_muon_ss, looked up once per device with that device current.
constexpr int kMaxDevices = 64;
float* g_ss_ptr[kMaxDevices] = {nullptr};
std::mutex g_mu;

cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ss_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_muon_ss);
    if (e != cudaSuccess) return e;
    g_ss_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_ss_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) cudaError_t br_muon_normalize_noalloc(
    const float* grad, float* mom, __nv_bfloat16* x_out, int S, int64_t n, float mu, cudaStream_t stream) {
  if (!grad || !mom || !x_out || S < 1 || S > BR_MUON_NOALLOC_MAX_MATRICES || n < 1) return cudaErrorInvalidValue;
  float* ss = nullptr;
  cudaError_t e = scratch_for_current_device(&ss);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  int64_t chunks = (n + 1023) / 1024;
  const int64_t cap = 4 * (int64_t)sms / S + 1;
  if (chunks > cap) chunks = cap;
  if (chunks < 1) chunks = 1;
  const dim3 grid((unsigned)chunks, (unsigned)S);
  // cudaLaunchKernel returns the status of this launch itself, so an error left on the thread by
  // earlier, unrelated work is neither reported as this call's failure nor cleared
  {
    void* args[] = {&ss, &S};
    if ((e = cudaLaunchKernel(reinterpret_cast<const void*>(noalloc_clear_kernel), dim3((S + 255) / 256), dim3(256),
                              args, 0, stream)) != cudaSuccess)
      return e;
  }
  {
    void* args[] = {const_cast<float**>(&grad), &mom, &n, &mu, &ss};
    if ((e = cudaLaunchKernel(reinterpret_cast<const void*>(noalloc_momentum_kernel), grid, dim3(256), args, 0,
                              stream)) != cudaSuccess)
      return e;
  }
  {
    const float* ssc = ss;
    void* args[] = {const_cast<float**>(&grad), &mom, &n, &mu, const_cast<float**>(&ssc), &x_out};
    e = cudaLaunchKernel(reinterpret_cast<const void*>(noalloc_normalize_kernel), grid, dim3(256), args, 0, stream);
  }
  return e;
}
