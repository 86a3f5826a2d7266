// Attention-input transforms, one warp per (token, head slot) over the fused QKV projection output
// qkv[M, H*hd + 2*KV*hd] (bf16, columns q | k | v):
//
//   q, k : half-split RoPE (y1 = x1 c + x2 s, y2 = -x1 s + x2 c, base 10000, gpt.ts:159-177) then
//          RMSNorm over head_dim (QK-norm after RoPE, gpt.ts:239-244); the per-head rstd is saved.
//   v    : value embedding on VE layers, v += ve[idx] * 2*sigmoid(cur[:, :32] @ Wg) where cur is the
//          un-normalised ladder output (gpt.ts:225-236); the gate is saved.
//
// Backward inverts each step: RMSNorm backward from the saved output and rstd, the transposed
// rotation, and for v the gate/table gradients (dve via vector reductions into the fp32 table grad,
// dz = dgate * gate * (1 - gate/2) stored per (token, kv head)). ``ve_gate_bwd`` turns dz into
// dWg = cur[:, :32]^T dz and the gradient flowing back into cur[:, :32].
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace br {
namespace {

constexpr float kEps = 1e-5f;
constexpr int kWarps = 8;
constexpr int kGateCh = 32;

struct RopeArgs {
  int M, T, H, KV, hd;
  int ld;  // row stride of qkv (elements)
};

__global__ void rope_fwd_kernel(__nv_bfloat16* __restrict__ qkv, RopeArgs a, const float* __restrict__ cosT,
                                const float* __restrict__ sinT, float* __restrict__ rq, float* __restrict__ rk,
                                const int* __restrict__ idx, const float* __restrict__ ve,
                                const float* __restrict__ cur, const float* __restrict__ wg, float* __restrict__ gate,
                                int D) {
  const int lane = threadIdx.x & 31;
  const int slots = a.H + 2 * a.KV;
  const int h2 = a.hd / 2;
  const int64_t total = (int64_t)a.M * slots;
  for (int64_t task = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5); task < total;
       task += (int64_t)gridDim.x * kWarps) {
    const int m = (int)(task / slots);
    const int s = (int)(task % slots);
    __nv_bfloat16* row = qkv + (int64_t)m * a.ld;
    if (s < a.H + a.KV) {
      const bool isq = s < a.H;
      const int head = isq ? s : s - a.H;
      __nv_bfloat16* p = row + (isq ? head * a.hd : a.H * a.hd + head * a.hd);
      const int t = m % a.T;
      float y1[4], y2[4];
      float ss = 0.f;
      int n = 0;
      for (int j = lane; j < h2; j += 32, ++n) {
        const float c = cosT[t * h2 + j], sn = sinT[t * h2 + j];
        const float x1 = __bfloat162float(p[j]), x2 = __bfloat162float(p[j + h2]);
        y1[n] = x1 * c + x2 * sn;
        y2[n] = -x1 * sn + x2 * c;
        ss += y1[n] * y1[n] + y2[n] * y2[n];
      }
      const float r = rsqrtf(warp_sum(ss) / a.hd + kEps);
      n = 0;
      for (int j = lane; j < h2; j += 32, ++n) {
        p[j] = __float2bfloat16(y1[n] * r);
        p[j + h2] = __float2bfloat16(y2[n] * r);
      }
      if (lane == 0) (isq ? rq[(int64_t)m * a.H + head] : rk[(int64_t)m * a.KV + head]) = r;
    } else if (ve != nullptr) {
      const int head = s - a.H - a.KV;
      float z = lane < kGateCh ? cur[(int64_t)m * D + lane] * wg[lane * a.KV + head] : 0.f;
      z = warp_sum(z);
      const float g = 2.f / (1.f + __expf(-z));
      __nv_bfloat16* p = row + a.H * a.hd + a.KV * a.hd + head * a.hd;
      const float* e = ve + (int64_t)idx[m] * (a.KV * a.hd) + head * a.hd;
      for (int j = lane; j < a.hd; j += 32) p[j] = __float2bfloat16(__bfloat162float(p[j]) + e[j] * g);
      if (lane == 0) gate[(int64_t)m * a.KV + head] = g;
    }
  }
}

// dqkv (in: grads of the transformed q,k,v; out: grads of the raw projection output), in place.
__global__ void rope_bwd_kernel(__nv_bfloat16* __restrict__ dqkv, const __nv_bfloat16* __restrict__ qkv, RopeArgs a,
                                const float* __restrict__ cosT, const float* __restrict__ sinT,
                                const float* __restrict__ rq, const float* __restrict__ rk,
                                const int* __restrict__ idx, const float* __restrict__ ve,
                                const float* __restrict__ gate, float* __restrict__ dve, float* __restrict__ dz) {
  const int lane = threadIdx.x & 31;
  const int slots = a.H + 2 * a.KV;
  const int h2 = a.hd / 2;
  const int64_t total = (int64_t)a.M * slots;
  for (int64_t task = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5); task < total;
       task += (int64_t)gridDim.x * kWarps) {
    const int m = (int)(task / slots);
    const int s = (int)(task % slots);
    if (s < a.H + a.KV) {
      const bool isq = s < a.H;
      const int head = isq ? s : s - a.H;
      const int64_t off = (int64_t)m * a.ld + (isq ? head * a.hd : a.H * a.hd + head * a.hd);
      const float r = isq ? rq[(int64_t)m * a.H + head] : rk[(int64_t)m * a.KV + head];
      float g1[4], g2[4], u1[4], u2[4];
      float dot = 0.f;
      int n = 0;
      for (int j = lane; j < h2; j += 32, ++n) {
        g1[n] = __bfloat162float(dqkv[off + j]);
        g2[n] = __bfloat162float(dqkv[off + j + h2]);
        u1[n] = __bfloat162float(qkv[off + j]);  // normalised outputs y
        u2[n] = __bfloat162float(qkv[off + j + h2]);
        dot += g1[n] * u1[n] + g2[n] * u2[n];
      }
      const float mean = warp_sum(dot) / a.hd;
      const int t = m % a.T;
      n = 0;
      for (int j = lane; j < h2; j += 32, ++n) {
        const float d1 = r * (g1[n] - u1[n] * mean), d2 = r * (g2[n] - u2[n] * mean);
        const float c = cosT[t * h2 + j], sn = sinT[t * h2 + j];
        dqkv[off + j] = __float2bfloat16(d1 * c - d2 * sn);
        dqkv[off + j + h2] = __float2bfloat16(d1 * sn + d2 * c);
      }
    } else if (ve != nullptr) {
      const int head = s - a.H - a.KV;
      const int64_t off = (int64_t)m * a.ld + a.H * a.hd + a.KV * a.hd + head * a.hd;
      const int64_t eoff = (int64_t)idx[m] * (a.KV * a.hd) + head * a.hd;
      const float g = gate[(int64_t)m * a.KV + head];
      float dg = 0.f;
      for (int j = lane * 4; j < a.hd; j += 128) {
        const float4 e = *reinterpret_cast<const float4*>(ve + eoff + j);
        const uint2 u = *reinterpret_cast<const uint2*>(dqkv + off + j);
        const float2 d01 = unpack_bf16(u.x), d23 = unpack_bf16(u.y);
        dg += d01.x * e.x + d01.y * e.y + d23.x * e.z + d23.y * e.w;
        red_add_v4_f32(dve + eoff + j, d01.x * g, d01.y * g, d23.x * g, d23.y * g);
      }
      dg = warp_sum(dg);
      if (lane == 0) dz[(int64_t)m * a.KV + head] = dg * g * (1.f - 0.5f * g);
    }
  }
}

// dWg[c,h] += sum_m cur[m,c] dz[m,h];  dgate_in[m,c] = sum_h dz[m,h] Wg[c,h]
template <int KVMAX>
__global__ void ve_gate_bwd_kernel(const float* __restrict__ cur, const float* __restrict__ dz,
                                   const float* __restrict__ wg, float* __restrict__ dwg, float* __restrict__ dgate_in,
                                   int M, int KV, int D) {
  __shared__ float red[kWarps][32][KVMAX];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float acc[KVMAX];
  float wrow[KVMAX];
#pragma unroll
  for (int h = 0; h < KVMAX; ++h) {
    acc[h] = 0.f;
    wrow[h] = h < KV ? wg[lane * KV + h] : 0.f;
  }
  for (int m = blockIdx.x * kWarps + w; m < M; m += gridDim.x * kWarps) {
    const float c = cur[(int64_t)m * D + lane];
    float gi = 0.f;
#pragma unroll
    for (int h = 0; h < KVMAX; ++h) {
      if (h < KV) {
        const float d = dz[(int64_t)m * KV + h];
        acc[h] += c * d;
        gi += d * wrow[h];
      }
    }
    dgate_in[(int64_t)m * kGateCh + lane] = gi;
  }
#pragma unroll
  for (int h = 0; h < KVMAX; ++h) red[w][lane][h] = acc[h];
  __syncthreads();
  if (w == 0) {
    for (int h = 0; h < KV; ++h) {
      float s = 0.f;
      for (int i = 0; i < kWarps; ++i) s += red[i][lane][h];
      atomicAdd(dwg + lane * KV + h, s);
    }
  }
}

int grid_for(int64_t tasks) {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int)std::max<int64_t>(1, std::min<int64_t>((tasks + kWarps - 1) / kWarps, (int64_t)sms * 16));
}

}  // namespace

void rope_fwd(torch::Tensor& qkv, int64_t T, int64_t H, int64_t KV, int64_t hd, const torch::Tensor& cosT,
              const torch::Tensor& sinT, torch::Tensor& rq, torch::Tensor& rk, const torch::Tensor& idx,
              c10::optional<torch::Tensor> ve, c10::optional<torch::Tensor> cur, c10::optional<torch::Tensor> wg,
              c10::optional<torch::Tensor> gate) {
  TORCH_CHECK(hd % 2 == 0 && hd <= 256 && hd % 4 == 0, "rope_fwd: head_dim must be a multiple of 4, <= 256");
  const int64_t M = qkv.size(0);
  RopeArgs a{(int)M, (int)T, (int)H, (int)KV, (int)hd, (int)qkv.stride(0)};
  const bool has_ve = ve.has_value() && ve->defined();
  c10::cuda::CUDAGuard g(qkv.device());
  const int64_t slots = H + (has_ve ? 2 : 1) * KV;
  rope_fwd_kernel<<<grid_for(M * slots), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), a, cosT.data_ptr<float>(), sinT.data_ptr<float>(),
      rq.data_ptr<float>(), rk.data_ptr<float>(), idx.data_ptr<int>(), has_ve ? ve->data_ptr<float>() : nullptr,
      has_ve ? cur->data_ptr<float>() : nullptr, has_ve ? wg->data_ptr<float>() : nullptr,
      has_ve ? gate->data_ptr<float>() : nullptr, has_ve ? (int)cur->size(-1) : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_bwd(torch::Tensor& dqkv, const torch::Tensor& qkv, int64_t T, int64_t H, int64_t KV, int64_t hd,
              const torch::Tensor& cosT, const torch::Tensor& sinT, const torch::Tensor& rq, const torch::Tensor& rk,
              const torch::Tensor& idx, c10::optional<torch::Tensor> ve, c10::optional<torch::Tensor> gate,
              c10::optional<torch::Tensor> dve, c10::optional<torch::Tensor> dz) {
  const int64_t M = qkv.size(0);
  TORCH_CHECK(dqkv.stride(0) == qkv.stride(0), "rope_bwd: dqkv/qkv row strides differ");
  RopeArgs a{(int)M, (int)T, (int)H, (int)KV, (int)hd, (int)qkv.stride(0)};
  const bool has_ve = ve.has_value() && ve->defined();
  c10::cuda::CUDAGuard g(qkv.device());
  const int64_t slots = H + (has_ve ? 2 : 1) * KV;
  rope_bwd_kernel<<<grid_for(M * slots), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), a,
      cosT.data_ptr<float>(), sinT.data_ptr<float>(), rq.data_ptr<float>(), rk.data_ptr<float>(), idx.data_ptr<int>(),
      has_ve ? ve->data_ptr<float>() : nullptr, has_ve ? gate->data_ptr<float>() : nullptr,
      has_ve ? dve->data_ptr<float>() : nullptr, has_ve ? dz->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ve_gate_bwd(const torch::Tensor& cur, const torch::Tensor& dz, const torch::Tensor& wg, torch::Tensor& dwg,
                 torch::Tensor& dgate_in) {
  const int64_t D = cur.size(-1), M = cur.numel() / D, KV = wg.size(1);
  TORCH_CHECK(KV <= 16 && wg.size(0) == kGateCh, "ve_gate_bwd: KV <= 16, Wg [32, KV]");
  c10::cuda::CUDAGuard g(cur.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = std::min(grid_for(M), 2 * 148);
  if (KV <= 4)
    ve_gate_bwd_kernel<4><<<grid, 32 * kWarps, 0, st>>>(cur.data_ptr<float>(), dz.data_ptr<float>(),
                                                         wg.data_ptr<float>(), dwg.data_ptr<float>(),
                                                         dgate_in.data_ptr<float>(), (int)M, (int)KV, (int)D);
  else
    ve_gate_bwd_kernel<16><<<grid, 32 * kWarps, 0, st>>>(cur.data_ptr<float>(), dz.data_ptr<float>(),
                                                          wg.data_ptr<float>(), dwg.data_ptr<float>(),
                                                          dgate_in.data_ptr<float>(), (int)M, (int)KV, (int)D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br
