// Attention-input transforms, one warp per token over the fused QKV projection output
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
#include "status.h"

namespace br {
namespace {

constexpr float kEps = 1e-5f;
constexpr int kWarps = 8;
constexpr int kGateCh = 32;

struct RopeArgs {
  int M, T, H, KV, hd;
  int ld;      // row stride of qkv (elements)
  int V;       // rows of the value-embedding table (token ids are checked against it)
  int* status;
};

// One warp per token; lane l owns head elements {2l, 2l+1} and {h2+2l, h2+2l+1} (hd = 128), so every
// load/store of the warp is a contiguous 128-byte bf16x2 access.
__device__ __forceinline__ float2 ldb2(const __nv_bfloat16* p) {
  return unpack_bf16(*reinterpret_cast<const uint32_t*>(p));
}
__device__ __forceinline__ void stb2(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16(a, b);
}

// The q/k heads of a token go in groups of G = 8: every head of a group is loaded before any is
// transformed, so a warp keeps a group's loads in flight and its warp reductions run side by side.
constexpr int G = 8;

__global__ void __launch_bounds__(256) rope_fwd_kernel(__nv_bfloat16* __restrict__ qkv, RopeArgs a,
                                                       const float* __restrict__ cosT, const float* __restrict__ sinT,
                                                       float* __restrict__ rq, float* __restrict__ rk,
                                                       const int* __restrict__ idx, const float* __restrict__ ve,
                                                       const float* __restrict__ cur, const float* __restrict__ wg,
                                                       float* __restrict__ gate, int D) {
  const int lane = threadIdx.x & 31;
  constexpr int h2 = 64;  // hd / 2
  const int nqk = a.H + a.KV;
  for (int m = blockIdx.x * kWarps + (threadIdx.x >> 5); m < a.M; m += gridDim.x * kWarps) {
    __nv_bfloat16* row = qkv + (int64_t)m * a.ld;
    const int t = m % a.T;
    const float2 c = *reinterpret_cast<const float2*>(cosT + t * h2 + 2 * lane);
    const float2 sn = *reinterpret_cast<const float2*>(sinT + t * h2 + 2 * lane);
    for (int s0 = 0; s0 < nqk; s0 += G) {
      __nv_bfloat16* hrow = row + s0 * 128;
      const int ng = min(G, nqk - s0);
      float2 x1[G], x2[G];
#pragma unroll
      for (int s = 0; s < G; ++s) {
        if (s < ng) {
          x1[s] = ldb2(hrow + s * 128 + 2 * lane);
          x2[s] = ldb2(hrow + s * 128 + h2 + 2 * lane);
        }
      }
      float ss[G];
#pragma unroll
      for (int s = 0; s < G; ++s) {
        ss[s] = 0.f;
        if (s < ng) {
          const float y1a = x1[s].x * c.x + x2[s].x * sn.x, y1b = x1[s].y * c.y + x2[s].y * sn.y;
          const float y2a = -x1[s].x * sn.x + x2[s].x * c.x, y2b = -x1[s].y * sn.y + x2[s].y * c.y;
          x1[s] = make_float2(y1a, y1b);
          x2[s] = make_float2(y2a, y2b);
          ss[s] = y1a * y1a + y1b * y1b + y2a * y2a + y2b * y2b;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int s = 0; s < G; ++s) ss[s] += __shfl_xor_sync(0xffffffffu, ss[s], o);
      }
#pragma unroll
      for (int s = 0; s < G; ++s) {
        if (s < ng) {
          const float r = rsqrtf(ss[s] / 128.f + kEps);
          stb2(hrow + s * 128 + 2 * lane, x1[s].x * r, x1[s].y * r);
          stb2(hrow + s * 128 + h2 + 2 * lane, x2[s].x * r, x2[s].y * r);
          const int hs = s0 + s;
          if (lane == s) (hs < a.H ? rq[(int64_t)m * a.H + hs] : rk[(int64_t)m * a.KV + (hs - a.H)]) = r;
        }
      }
    }
    if (ve != nullptr && index_ok(idx[m], a.V, lane == 0 ? a.status : nullptr)) {
      const float cz = cur[(int64_t)m * D + lane];
      const float* e = ve + (int64_t)idx[m] * (a.KV * 128);
      for (int h = 0; h < a.KV; ++h) {
        const float z = warp_sum(cz * wg[lane * a.KV + h]);
        const float g = 2.f / (1.f + __expf(-z));
        __nv_bfloat16* p = row + (nqk + h) * 128;
        const float4 ev = *reinterpret_cast<const float4*>(e + h * 128 + 4 * lane);
        const uint2 u = *reinterpret_cast<const uint2*>(p + 4 * lane);
        const float2 v01 = unpack_bf16(u.x), v23 = unpack_bf16(u.y);
        uint2 o;
        o.x = pack_bf16(v01.x + ev.x * g, v01.y + ev.y * g);
        o.y = pack_bf16(v23.x + ev.z * g, v23.y + ev.w * g);
        *reinterpret_cast<uint2*>(p + 4 * lane) = o;
        if (lane == 0) gate[(int64_t)m * a.KV + h] = g;
      }
    }
  }
}

// dqkv (in: grads of the transformed q,k,v; out: grads of the raw projection output), in place.
__global__ void __launch_bounds__(256) rope_bwd_kernel(__nv_bfloat16* __restrict__ dqkv,
                                                       const __nv_bfloat16* __restrict__ qkv, RopeArgs a,
                                                       const float* __restrict__ cosT, const float* __restrict__ sinT,
                                                       const float* __restrict__ rq, const float* __restrict__ rk,
                                                       const int* __restrict__ idx, const float* __restrict__ ve,
                                                       const float* __restrict__ gate, float* __restrict__ dve,
                                                       float* __restrict__ dz) {
  const int lane = threadIdx.x & 31;
  constexpr int h2 = 64;
  const int nqk = a.H + a.KV;
  for (int m = blockIdx.x * kWarps + (threadIdx.x >> 5); m < a.M; m += gridDim.x * kWarps) {
    const int64_t base = (int64_t)m * a.ld;
    const int t = m % a.T;
    const float2 c = *reinterpret_cast<const float2*>(cosT + t * h2 + 2 * lane);
    const float2 sn = *reinterpret_cast<const float2*>(sinT + t * h2 + 2 * lane);
    // lane s < nqk fetches head s's rstd; it is broadcast below
    const float rl = lane < a.H ? rq[(int64_t)m * a.H + lane]
                                : (lane < nqk ? rk[(int64_t)m * a.KV + (lane - a.H)] : 0.f);
    for (int s0 = 0; s0 < nqk; s0 += G) {
      const int ng = min(G, nqk - s0);
      float2 g1[G], g2[G], u1[G], u2[G];
#pragma unroll
      for (int s = 0; s < G; ++s) {
        if (s < ng) {
          const int64_t off = base + (s0 + s) * 128;
          g1[s] = ldb2(dqkv + off + 2 * lane);
          g2[s] = ldb2(dqkv + off + h2 + 2 * lane);
          u1[s] = ldb2(qkv + off + 2 * lane);
          u2[s] = ldb2(qkv + off + h2 + 2 * lane);
        }
      }
      float dot[G];
#pragma unroll
      for (int s = 0; s < G; ++s)
        dot[s] = s < ng ? g1[s].x * u1[s].x + g1[s].y * u1[s].y + g2[s].x * u2[s].x + g2[s].y * u2[s].y : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int s = 0; s < G; ++s) dot[s] += __shfl_xor_sync(0xffffffffu, dot[s], o);
      }
#pragma unroll
      for (int s = 0; s < G; ++s) {
        const float r = __shfl_sync(0xffffffffu, rl, s0 + s);  // every lane shuffles (full mask)
        if (s < ng) {
          const int64_t off = base + (s0 + s) * 128;
          const float mean = dot[s] / 128.f;
          const float d1a = r * (g1[s].x - u1[s].x * mean), d1b = r * (g1[s].y - u1[s].y * mean);
          const float d2a = r * (g2[s].x - u2[s].x * mean), d2b = r * (g2[s].y - u2[s].y * mean);
          stb2(dqkv + off + 2 * lane, d1a * c.x - d2a * sn.x, d1b * c.y - d2b * sn.y);
          stb2(dqkv + off + h2 + 2 * lane, d1a * sn.x + d2a * c.x, d1b * sn.y + d2b * c.y);
        }
      }
    }
    if (ve != nullptr && !index_ok(idx[m], a.V, lane == 0 ? a.status : nullptr)) {
      if (lane < a.KV) dz[(int64_t)m * a.KV + lane] = 0.f;  // the forward skipped this row's VE add
    } else if (ve != nullptr) {
      const int64_t erow = (int64_t)idx[m] * (a.KV * 128);
      for (int h = 0; h < a.KV; ++h) {
        const int64_t off = base + (nqk + h) * 128 + 4 * lane;
        const float g = gate[(int64_t)m * a.KV + h];
        const float4 e = *reinterpret_cast<const float4*>(ve + erow + h * 128 + 4 * lane);
        const uint2 u = *reinterpret_cast<const uint2*>(dqkv + off);
        const float2 d01 = unpack_bf16(u.x), d23 = unpack_bf16(u.y);
        const float dg = warp_sum(d01.x * e.x + d01.y * e.y + d23.x * e.z + d23.y * e.w);
        red_add_v4_f32(dve + erow + h * 128 + 4 * lane, d01.x * g, d01.y * g, d23.x * g, d23.y * g);
        if (lane == 0) dz[(int64_t)m * a.KV + h] = dg * g * (1.f - 0.5f * g);
      }
    }
  }
}

// 64-wide heads: one warp per token, one head at a time. Lane l < 16 holds elements 2l, 2l+1 of the first
// half of the head and lane l + 16 the same elements of the second half, so RoPE's partner values are one
// shuffle away (xor 16); the cos/sin tables are [T, 32].
__global__ void __launch_bounds__(256) rope64_fwd_kernel(__nv_bfloat16* __restrict__ qkv, RopeArgs a,
                                                         const float* __restrict__ cosT, const float* __restrict__ sinT,
                                                         float* __restrict__ rq, float* __restrict__ rk,
                                                         const int* __restrict__ idx, const float* __restrict__ ve,
                                                         const float* __restrict__ cur, const float* __restrict__ wg,
                                                         float* __restrict__ gate, int D) {
  const int lane = threadIdx.x & 31;
  const bool first = lane < 16;
  const int nqk = a.H + a.KV;
  for (int m = blockIdx.x * kWarps + (threadIdx.x >> 5); m < a.M; m += gridDim.x * kWarps) {
    __nv_bfloat16* row = qkv + (int64_t)m * a.ld;
    const int t = m % a.T;
    const float2 c = *reinterpret_cast<const float2*>(cosT + t * 32 + 2 * (lane & 15));
    const float2 sn = *reinterpret_cast<const float2*>(sinT + t * 32 + 2 * (lane & 15));
    for (int hs = 0; hs < nqk; ++hs) {
      __nv_bfloat16* hp = row + hs * 64 + 2 * lane;
      const float2 x = ldb2(hp);
      const float2 q = make_float2(__shfl_xor_sync(0xffffffffu, x.x, 16), __shfl_xor_sync(0xffffffffu, x.y, 16));
      // first half: y1 = x1 c + x2 s; second half: y2 = x2 c - x1 s
      const float sg = first ? 1.f : -1.f;
      const float ya = x.x * c.x + sg * q.x * sn.x, yb = x.y * c.y + sg * q.y * sn.y;
      const float r = rsqrtf(warp_sum(ya * ya + yb * yb) / 64.f + kEps);
      stb2(hp, ya * r, yb * r);
      if (lane == 0) (hs < a.H ? rq[(int64_t)m * a.H + hs] : rk[(int64_t)m * a.KV + (hs - a.H)]) = r;
    }
    if (ve != nullptr && index_ok(idx[m], a.V, lane == 0 ? a.status : nullptr)) {
      const float cz = cur[(int64_t)m * D + lane];
      const float* e = ve + (int64_t)idx[m] * (a.KV * 64);
      for (int h = 0; h < a.KV; ++h) {
        const float z = warp_sum(cz * wg[lane * a.KV + h]);
        const float g = 2.f / (1.f + __expf(-z));
        __nv_bfloat16* pv = row + (nqk + h) * 64 + 2 * lane;
        const float2 ev = *reinterpret_cast<const float2*>(e + h * 64 + 2 * lane);
        const float2 v = ldb2(pv);
        stb2(pv, v.x + ev.x * g, v.y + ev.y * g);
        if (lane == 0) gate[(int64_t)m * a.KV + h] = g;
      }
    }
  }
}

// Backward of rope64_fwd_kernel, in place on dqkv (qkv holds the forward's normalised outputs).
__global__ void __launch_bounds__(256) rope64_bwd_kernel(__nv_bfloat16* __restrict__ dqkv,
                                                         const __nv_bfloat16* __restrict__ qkv, RopeArgs a,
                                                         const float* __restrict__ cosT, const float* __restrict__ sinT,
                                                         const float* __restrict__ rq, const float* __restrict__ rk,
                                                         const int* __restrict__ idx, const float* __restrict__ ve,
                                                         const float* __restrict__ gate, float* __restrict__ dve,
                                                         float* __restrict__ dz) {
  const int lane = threadIdx.x & 31;
  const bool first = lane < 16;
  const int nqk = a.H + a.KV;
  for (int m = blockIdx.x * kWarps + (threadIdx.x >> 5); m < a.M; m += gridDim.x * kWarps) {
    const int64_t base = (int64_t)m * a.ld;
    const int t = m % a.T;
    const float2 c = *reinterpret_cast<const float2*>(cosT + t * 32 + 2 * (lane & 15));
    const float2 sn = *reinterpret_cast<const float2*>(sinT + t * 32 + 2 * (lane & 15));
    for (int hs = 0; hs < nqk; ++hs) {
      const int64_t off = base + hs * 64 + 2 * lane;
      const float r = hs < a.H ? rq[(int64_t)m * a.H + hs] : rk[(int64_t)m * a.KV + (hs - a.H)];
      const float2 g = ldb2(dqkv + off), u = ldb2(qkv + off);
      const float mean = warp_sum(g.x * u.x + g.y * u.y) / 64.f;
      // gradient of the rotated (pre-norm) values, then the inverse rotation:
      // dx1 = dy1 c - dy2 s (first half), dx2 = dy2 c + dy1 s (second half)
      const float da = r * (g.x - u.x * mean), db = r * (g.y - u.y * mean);
      const float pa = __shfl_xor_sync(0xffffffffu, da, 16), pb = __shfl_xor_sync(0xffffffffu, db, 16);
      const float sg = first ? -1.f : 1.f;
      stb2(dqkv + off, da * c.x + sg * pa * sn.x, db * c.y + sg * pb * sn.y);
    }
    if (ve != nullptr && !index_ok(idx[m], a.V, lane == 0 ? a.status : nullptr)) {
      if (lane < a.KV) dz[(int64_t)m * a.KV + lane] = 0.f;  // the forward skipped this row's VE add
    } else if (ve != nullptr) {
      const int64_t erow = (int64_t)idx[m] * (a.KV * 64);
      for (int h = 0; h < a.KV; ++h) {
        const int64_t off = base + (nqk + h) * 64 + 2 * lane;
        const float g = gate[(int64_t)m * a.KV + h];
        const float2 e = *reinterpret_cast<const float2*>(ve + erow + h * 64 + 2 * lane);
        const float2 d = ldb2(dqkv + off);
        const float dg = warp_sum(d.x * e.x + d.y * e.y);
        atomicAdd(dve + erow + h * 64 + 2 * lane, d.x * g);
        atomicAdd(dve + erow + h * 64 + 2 * lane + 1, d.y * g);
        if (lane == 0) dz[(int64_t)m * a.KV + h] = dg * g * (1.f - 0.5f * g);
      }
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
  return (int)std::max<int64_t>(1, std::min<int64_t>((tasks + kWarps - 1) / kWarps, (int64_t)sms * 8));
}

}  // namespace

void rope_fwd(torch::Tensor& qkv, int64_t T, int64_t H, int64_t KV, int64_t hd, const torch::Tensor& cosT,
              const torch::Tensor& sinT, torch::Tensor& rq, torch::Tensor& rk, const torch::Tensor& idx,
              c10::optional<torch::Tensor> ve, c10::optional<torch::Tensor> cur, c10::optional<torch::Tensor> wg,
              c10::optional<torch::Tensor> gate) {
  TORCH_CHECK(hd == 128 || hd == 64, "rope_fwd: head_dim 64 or 128");
  TORCH_CHECK(qkv.stride(0) % 8 == 0, "rope_fwd: row stride must be a multiple of 8");
  const int64_t M = qkv.size(0);
  const bool has_ve = ve.has_value() && ve->defined();
  RopeArgs a{(int)M, (int)T, (int)H, (int)KV, (int)hd, (int)qkv.stride(0), has_ve ? (int)ve->size(0) : 0,
             status_ptr(qkv.device().index())};
  c10::cuda::CUDAGuard g(qkv.device());
  TORCH_CHECK(H + KV <= 32, "rope_fwd: at most 32 q/k heads");
  auto kern = hd == 128 ? rope_fwd_kernel : rope64_fwd_kernel;
  kern<<<grid_for(M), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
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
  const bool has_ve = ve.has_value() && ve->defined();
  RopeArgs a{(int)M, (int)T, (int)H, (int)KV, (int)hd, (int)qkv.stride(0), has_ve ? (int)ve->size(0) : 0,
             status_ptr(qkv.device().index())};
  c10::cuda::CUDAGuard g(qkv.device());
  TORCH_CHECK((hd == 128 || hd == 64) && H + KV <= 32, "rope_bwd: head_dim 64 or 128, at most 32 q/k heads");
  auto kern = hd == 128 ? rope_bwd_kernel : rope64_bwd_kernel;
  kern<<<grid_for(M), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
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
