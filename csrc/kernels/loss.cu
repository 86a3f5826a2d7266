// Fused cross-entropy over softcapped logits (gpt.ts:302-313), forward and backward in one pass.
//
// Input: logits l = cap*tanh(z/cap) in bf16 [M, V] (written by the lm_head GEMM's softcap
// epilogue). Per row, with t = target (ignored when -1):
//   p = softmax(l),  nats = -log(p_t + 1e-10)          (the reference's eps form, not log-softmax)
//   loss += valid * nats * scale                        (scale = 1/(B*T): mean over all positions)
//   dz_j = valid*scale * p_t/(p_t+1e-10) * (p_j - [j==t]) * (1 - (l_j/cap)^2)
// dz (the gradient w.r.t. the pre-softcap GEMM output) overwrites the logits in place as bf16.
// One 256-thread block per row: an online max/sum pass, then the gradient pass (second read from L1).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace br {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void online(float& m, float& s, float x) {
  if (x > m) {
    s = s * __expf(m - x) + 1.f;
    m = x;
  } else {
    s += __expf(x - m);
  }
}

template <bool GRAD>
__global__ void __launch_bounds__(kThreads) ce_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld,
                                                       const int* __restrict__ targets, int V, float cap, float scale,
                                                       float* __restrict__ nats, float* __restrict__ loss_sum) {
  __shared__ float sm[kThreads / 32], ss[kThreads / 32];
  __shared__ float bcast[3];
  const int row = blockIdx.x;
  __nv_bfloat16* L = logits + (int64_t)row * ld;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float m = -INFINITY, s = 0.f;
  const int nvec = V / 8;
  for (int i = threadIdx.x; i < nvec; i += kThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(L + i * 8);
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16(q[k]);
      online(m, s, f.x);
      online(m, s, f.y);
    }
  }
  for (int j = nvec * 8 + threadIdx.x; j < V; j += kThreads) online(m, s, __bfloat162float(L[j]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffff, m, o), s2 = __shfl_xor_sync(0xffffffff, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  if (lane == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int i = 1; i < kThreads / 32; ++i) {
      const float mm = fmaxf(M, sm[i]);
      S = S * __expf(M - mm) + ss[i] * __expf(sm[i] - mm);
      M = mm;
    }
    const int t = targets[row];
    const int tt = t < 0 ? 0 : t;
    const float pt = __expf(__bfloat162float(L[tt]) - M) / S;
    const float nll = -__logf(pt + 1e-10f);
    if (nats) nats[row] = nll;
    const float valid = t == -1 ? 0.f : 1.f;
    if (loss_sum) atomicAdd(loss_sum, valid * nll * scale);
    const float coef = valid * scale * (pt / (pt + 1e-10f));
    bcast[0] = M;
    bcast[1] = coef / S;
    bcast[2] = coef;
  }
  __syncthreads();
  if constexpr (GRAD) {
    const float M = bcast[0], cs = bcast[1], coef = bcast[2];
    const int t = targets[row];
    const float ic = 1.f / cap;
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      const uint4 u = *reinterpret_cast<const uint4*>(L + i * 8);
      uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16(q[k]);
        const int j0 = i * 8 + 2 * k;
        float g0 = __expf(f.x - M) * cs - (j0 == t ? coef : 0.f);
        float g1 = __expf(f.y - M) * cs - (j0 + 1 == t ? coef : 0.f);
        g0 *= 1.f - (f.x * ic) * (f.x * ic);
        g1 *= 1.f - (f.y * ic) * (f.y * ic);
        q[k] = pack_bf16(g0, g1);
      }
      *reinterpret_cast<uint4*>(L + i * 8) = make_uint4(q[0], q[1], q[2], q[3]);
    }
    for (int j = nvec * 8 + threadIdx.x; j < V; j += kThreads) {
      const float l = __bfloat162float(L[j]);
      const float g = (__expf(l - M) * cs - (j == t ? coef : 0.f)) * (1.f - (l * ic) * (l * ic));
      L[j] = __float2bfloat16(g);
    }
  }
}

}  // namespace

// logits: bf16 [M, V] (row stride ld), softcapped; overwritten by dz when grad=true.
void softcap_ce(torch::Tensor& logits, const torch::Tensor& targets, double cap, double scale,
                c10::optional<torch::Tensor> nats, c10::optional<torch::Tensor> loss_sum, bool grad) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "softcap_ce: logits");
  TORCH_CHECK(targets.scalar_type() == at::kInt && targets.is_contiguous(), "softcap_ce: int32 targets");
  const int64_t M = logits.size(0), V = logits.size(1);
  TORCH_CHECK(logits.stride(0) % 8 == 0, "softcap_ce: row stride must be a multiple of 8");
  c10::cuda::CUDAGuard g(logits.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto* L = reinterpret_cast<__nv_bfloat16*>(logits.data_ptr());
  float* n = nats.has_value() ? nats->data_ptr<float>() : nullptr;
  float* ls = loss_sum.has_value() ? loss_sum->data_ptr<float>() : nullptr;
  if (grad)
    ce_kernel<true><<<(unsigned)M, kThreads, 0, st>>>(L, logits.stride(0), targets.data_ptr<int>(), (int)V,
                                                       (float)cap, (float)scale, n, ls);
  else
    ce_kernel<false><<<(unsigned)M, kThreads, 0, st>>>(L, logits.stride(0), targets.data_ptr<int>(), (int)V,
                                                        (float)cap, (float)scale, n, ls);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br
