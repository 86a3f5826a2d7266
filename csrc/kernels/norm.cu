// Row kernels around RMSNorm (no weight, eps 1e-5, src/model/gpt.ts:146-152), one warp per row,
// 16-byte vector accesses, fp32 math:
//
//   embed_rms_fwd     x0 = rms(wte[idx])                               (gpt.ts:193-195)
//   ladder_rms_fwd    cur = lr[i]*x + l0[i]*x0 ; xn = bf16(rms(cur))    (gpt.ts:208-214)
//   rms_fwd           xn = bf16(rms(x))                                 (gpt.ts:286, 296)
//   rms_bwd           dx = rms'(x)^T dy (+ dres), fp32 and optional bf16 copy
//   ladder_bwd        dcur = rms'(cur)^T dxn + dres (+ VE-gate input grad on the first 32 columns);
//                     dx = lr*dcur, dx0 += l0*dcur, dlr[i] += <dcur, x>, dl0[i] += <dcur, x0>
//   embed_bwd         dwte[idx] += rms'(wte[idx])^T dx0                  (scatter with vector reductions)
//
// The scalar-lambda gradients are reduced per block and added with one atomic per block
// (grid-stride loops over rows keep the block count near a few per SM).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "status.h"

namespace br {
namespace {

constexpr float kEps = 1e-5f;
constexpr int kWarps = 8;

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ float4 ldb4(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void stb4(__nv_bfloat16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16(v.x, v.y);
  u.y = pack_bf16(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }
__device__ __forceinline__ float4 axpby4(float a, float4 x, float b, float4 y) {
  return make_float4(a * x.x + b * y.x, a * x.y + b * y.y, a * x.z + b * y.z, a * x.w + b * y.w);
}
__device__ __forceinline__ float4 scale4(float4 x, float s) { return make_float4(x.x * s, x.y * s, x.z * s, x.w * s); }

template <typename T>
__device__ __forceinline__ float4 load_any(const T* p);
template <>
__device__ __forceinline__ float4 load_any<float>(const float* p) { return ld4(p); }
template <>
__device__ __forceinline__ float4 load_any<__nv_bfloat16>(const __nv_bfloat16* p) { return ldb4(p); }

__global__ void embed_rms_fwd_kernel(const int* __restrict__ idx, const float* __restrict__ wte, float* __restrict__ x0,
                                     float* __restrict__ rstd, int M, int D, int V, int* status) {
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < M; row += gridDim.x * kWarps) {
    const int id = idx[row];
    if (!index_ok(id, V, lane == 0 ? status : nullptr)) {  // a zero row with rstd 0: no gradient either
      for (int c = lane * 4; c < D; c += 128) st4(x0 + (int64_t)row * D + c, make_float4(0.f, 0.f, 0.f, 0.f));
      if (lane == 0) rstd[row] = 0.f;
      continue;
    }
    const float* w = wte + (int64_t)id * D;
    float ss = 0.f;
    for (int c = lane * 4; c < D; c += 128) {
      float4 v = ld4(w + c);
      ss += dot4(v, v);
    }
    const float r = rsqrtf(warp_sum(ss) / D + kEps);
    float* o = x0 + (int64_t)row * D;
    for (int c = lane * 4; c < D; c += 128) st4(o + c, scale4(ld4(w + c), r));
    if (lane == 0) rstd[row] = r;
  }
}

__global__ void ladder_rms_fwd_kernel(const float* __restrict__ x, const float* __restrict__ x0,
                                      const float* __restrict__ lam_r, const float* __restrict__ lam_0, int layer,
                                      float* __restrict__ cur, __nv_bfloat16* __restrict__ xn, float* __restrict__ rstd,
                                      int M, int D) {
  const int lane = threadIdx.x & 31;
  const float a = lam_r[layer], b = lam_0[layer];
  for (int row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < M; row += gridDim.x * kWarps) {
    const int64_t off = (int64_t)row * D;
    float ss = 0.f;
    for (int c = lane * 4; c < D; c += 128) {
      float4 v = axpby4(a, ld4(x + off + c), b, ld4(x0 + off + c));
      st4(cur + off + c, v);
      ss += dot4(v, v);
    }
    const float r = rsqrtf(warp_sum(ss) / D + kEps);
    for (int c = lane * 4; c < D; c += 128) stb4(xn + off + c, scale4(ld4(cur + off + c), r));
    if (lane == 0) rstd[row] = r;
  }
}

__global__ void rms_fwd_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ xn, float* __restrict__ rstd,
                               int M, int D) {
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < M; row += gridDim.x * kWarps) {
    const int64_t off = (int64_t)row * D;
    float ss = 0.f;
    for (int c = lane * 4; c < D; c += 128) {
      float4 v = ld4(x + off + c);
      ss += dot4(v, v);
    }
    const float r = rsqrtf(warp_sum(ss) / D + kEps);
    for (int c = lane * 4; c < D; c += 128) stb4(xn + off + c, scale4(ld4(x + off + c), r));
    if (rstd && lane == 0) rstd[row] = r;
  }
}

// The lm_head backward's row terms (the fused softcapped cross-entropy, loss.cu): the incoming gradient
// is rowscale[row] * dy + coef[row] * w[targets[row]] (w: the [V, D] fp32 table; masked rows have
// coef 0 and a target outside [0, V)).
struct HeadGrad {
  const float* rowscale;
  const float* coef;
  const int* targets;
  const float* w;
  int V;
};

template <typename TD, bool HEAD>
__device__ __forceinline__ float4 head_dy(const TD* dy, int64_t off, int c, float rs, float cf, const float* wrow) {
  float4 g = load_any<TD>(dy + off + c);
  if constexpr (HEAD) {
    g = scale4(g, rs);
    if (wrow) g = axpby4(1.f, g, cf, ld4(wrow + c));
  }
  return g;
}

// dx = r * (dy - y * mean(dy*y)) + dres, y = x*r
template <typename TD, bool HEAD>
__global__ void rms_bwd_kernel(const float* __restrict__ x, const float* __restrict__ rstd, const TD* __restrict__ dy,
                               const float* __restrict__ dres, float* __restrict__ dx, __nv_bfloat16* __restrict__ dxb,
                               int M, int D, HeadGrad hg) {
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < M; row += gridDim.x * kWarps) {
    const int64_t off = (int64_t)row * D;
    const float r = rstd[row];
    float rs = 1.f, cf = 0.f;
    const float* wrow = nullptr;
    if constexpr (HEAD) {
      rs = hg.rowscale[row];
      if (hg.coef) {  // exact fp32 target form; without coef the target column is already inside dy
        cf = hg.coef[row];
        const int t = hg.targets[row];
        if (t >= 0 && t < hg.V) wrow = hg.w + (int64_t)t * D;
      }
    }
    float s = 0.f;
    for (int c = lane * 4; c < D; c += 128)
      s += dot4(head_dy<TD, HEAD>(dy, off, c, rs, cf, wrow), scale4(ld4(x + off + c), r));
    const float mean = warp_sum(s) / D;
    for (int c = lane * 4; c < D; c += 128) {
      float4 g = head_dy<TD, HEAD>(dy, off, c, rs, cf, wrow);
      float4 y = scale4(ld4(x + off + c), r);
      float4 o = make_float4(r * (g.x - y.x * mean), r * (g.y - y.y * mean), r * (g.z - y.z * mean),
                             r * (g.w - y.w * mean));
      if (dres) {
        float4 d = ld4(dres + off + c);
        o.x += d.x;
        o.y += d.y;
        o.z += d.z;
        o.w += d.w;
      }
      if (dx) st4(dx + off + c, o);
      if (dxb) stb4(dxb + off + c, o);
    }
  }
}

// dcur = r*(dxn - y*mean(dxn*y)) + dres (+ dgate on cols < 32); cur recomputed from x, x0.
template <typename TD>
__global__ void ladder_bwd_kernel(const float* __restrict__ x, const float* __restrict__ x0,
                                  const float* __restrict__ lam_r, const float* __restrict__ lam_0, int layer,
                                  const float* __restrict__ rstd, const TD* __restrict__ dxn,
                                  const float* __restrict__ dres, const float* __restrict__ dgate_in,
                                  float* __restrict__ dx, float* __restrict__ dx0_acc, float* __restrict__ dlam_r,
                                  float* __restrict__ dlam_0, int M, int D, int first_layer,
                                  __nv_bfloat16* __restrict__ dx_b) {
  __shared__ float red[2][kWarps];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float a = lam_r[layer], b = lam_0[layer];
  float acc_r = 0.f, acc_0 = 0.f;
  for (int row = blockIdx.x * kWarps + w; row < M; row += gridDim.x * kWarps) {
    const int64_t off = (int64_t)row * D;
    const float r = rstd[row];
    float s = 0.f;
    for (int c = lane * 4; c < D; c += 128) {
      float4 cur = axpby4(a, ld4(x + off + c), b, ld4(x0 + off + c));
      s += dot4(load_any<TD>(dxn + off + c), scale4(cur, r));
    }
    const float mean = warp_sum(s) / D;
    for (int c = lane * 4; c < D; c += 128) {
      float4 xi = ld4(x + off + c), x0i = ld4(x0 + off + c);
      float4 cur = axpby4(a, xi, b, x0i);
      float4 g = load_any<TD>(dxn + off + c);
      float4 y = scale4(cur, r);
      float4 d = make_float4(r * (g.x - y.x * mean), r * (g.y - y.y * mean), r * (g.z - y.z * mean),
                             r * (g.w - y.w * mean));
      float4 dr = ld4(dres + off + c);
      d.x += dr.x;
      d.y += dr.y;
      d.z += dr.z;
      d.w += dr.w;
      if (dgate_in && c < 32) {
        float4 gg = ld4(dgate_in + (int64_t)row * 32 + c);
        d.x += gg.x;
        d.y += gg.y;
        d.z += gg.z;
        d.w += gg.w;
      }
      acc_r += dot4(d, xi);
      acc_0 += dot4(d, x0i);
      float4 dxa = scale4(d, a);
      float4 acc = ld4(dx0_acc + off + c);
      float4 add0 = scale4(d, b);
      if (first_layer) {  // x == x0 at the first layer: both paths feed dx0
        add0.x += dxa.x;
        add0.y += dxa.y;
        add0.z += dxa.z;
        add0.w += dxa.w;
      } else {
        st4(dx + off + c, dxa);
        if (dx_b)  // the bf16 copy the previous layer's GEMMs read
          *reinterpret_cast<uint2*>(dx_b + off + c) = make_uint2(pack_bf16(dxa.x, dxa.y), pack_bf16(dxa.z, dxa.w));
      }
      st4(dx0_acc + off + c, make_float4(acc.x + add0.x, acc.y + add0.y, acc.z + add0.z, acc.w + add0.w));
    }
  }
  acc_r = warp_sum(acc_r);
  acc_0 = warp_sum(acc_0);
  if (lane == 0) {
    red[0][w] = acc_r;
    red[1][w] = acc_0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sr = 0.f, s0 = 0.f;
    for (int i = 0; i < kWarps; ++i) {
      sr += red[0][i];
      s0 += red[1][i];
    }
    atomicAdd(dlam_r + layer, sr);
    atomicAdd(dlam_0 + layer, s0);
  }
}

__global__ void embed_bwd_kernel(const int* __restrict__ idx, const float* __restrict__ wte,
                                 const float* __restrict__ rstd, const float* __restrict__ dx0, float* __restrict__ dwte,
                                 int M, int D, int V, int* status) {
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < M; row += gridDim.x * kWarps) {
    const int64_t off = (int64_t)row * D;
    const int id = idx[row];
    if (!index_ok(id, V, lane == 0 ? status : nullptr)) continue;
    const int64_t woff = (int64_t)id * D;
    const float r = rstd[row];
    float s = 0.f;
    for (int c = lane * 4; c < D; c += 128) s += dot4(ld4(dx0 + off + c), scale4(ld4(wte + woff + c), r));
    const float mean = warp_sum(s) / D;
    for (int c = lane * 4; c < D; c += 128) {
      float4 g = ld4(dx0 + off + c);
      float4 y = scale4(ld4(wte + woff + c), r);
      red_add_v4_f32(dwte + woff + c, r * (g.x - y.x * mean), r * (g.y - y.y * mean), r * (g.z - y.z * mean),
                     r * (g.w - y.w * mean));
    }
  }
}

__global__ void cast_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x)
    stb4(y + 4 * i, ld4(x + 4 * i));
}

int rows_grid(int64_t M) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (M + kWarps - 1) / kWarps;
  return (int)std::min<int64_t>(blocks, (int64_t)sms * 8);
}

void check_rows(const torch::Tensor& t, int64_t M, int64_t D, at::ScalarType st, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == st, name, ": bad tensor (device/layout/dtype)");
  TORCH_CHECK(t.numel() == M * D, name, ": bad size");
}

}  // namespace

void embed_rms_fwd(const torch::Tensor& idx, const torch::Tensor& wte, torch::Tensor& x0, torch::Tensor& rstd) {
  const int64_t M = idx.numel(), D = wte.size(1);
  TORCH_CHECK(D % 4 == 0 && idx.scalar_type() == at::kInt, "embed_rms_fwd: D%4 / int32 idx");
  check_rows(x0, M, D, at::kFloat, "x0");
  c10::cuda::CUDAGuard g(wte.device());
  embed_rms_fwd_kernel<<<rows_grid(M), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int>(), wte.data_ptr<float>(), x0.data_ptr<float>(), rstd.data_ptr<float>(), (int)M, (int)D,
      (int)wte.size(0), status_ptr(wte.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ladder_rms_fwd(const torch::Tensor& x, const torch::Tensor& x0, const torch::Tensor& lam_r,
                    const torch::Tensor& lam_0, int64_t layer, torch::Tensor& cur, torch::Tensor& xn,
                    torch::Tensor& rstd) {
  const int64_t D = x.size(-1), M = x.numel() / D;
  check_rows(cur, M, D, at::kFloat, "cur");
  check_rows(xn, M, D, at::kBFloat16, "xn");
  c10::cuda::CUDAGuard g(x.device());
  ladder_rms_fwd_kernel<<<rows_grid(M), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), x0.data_ptr<float>(), lam_r.data_ptr<float>(), lam_0.data_ptr<float>(), (int)layer,
      cur.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(xn.data_ptr()), rstd.data_ptr<float>(), (int)M, (int)D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rms_fwd(const torch::Tensor& x, torch::Tensor& xn, c10::optional<torch::Tensor> rstd) {
  const int64_t D = x.size(-1), M = x.numel() / D;
  check_rows(xn, M, D, at::kBFloat16, "xn");
  c10::cuda::CUDAGuard g(x.device());
  rms_fwd_kernel<<<rows_grid(M), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(xn.data_ptr()),
      rstd.has_value() ? rstd->data_ptr<float>() : nullptr, (int)M, (int)D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rms_bwd(const torch::Tensor& x, const torch::Tensor& rstd, const torch::Tensor& dy,
             c10::optional<torch::Tensor> dres, c10::optional<torch::Tensor> dx, c10::optional<torch::Tensor> dxb,
             c10::optional<torch::Tensor> rowscale, c10::optional<torch::Tensor> coef,
             c10::optional<torch::Tensor> targets, c10::optional<torch::Tensor> wtab) {
  const int64_t D = x.size(-1), M = x.numel() / D;
  TORCH_CHECK(D % 4 == 0, "rms_bwd: D % 4");
  c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const float* dr = dres.has_value() ? dres->data_ptr<float>() : nullptr;
  float* o = dx.has_value() ? dx->data_ptr<float>() : nullptr;
  __nv_bfloat16* ob = dxb.has_value() ? reinterpret_cast<__nv_bfloat16*>(dxb->data_ptr()) : nullptr;
  HeadGrad hg{};
  const bool head = rowscale.has_value() && rowscale->defined();
  if (head) {
    check_rows(*rowscale, M, 1, at::kFloat, "rowscale");
    hg.rowscale = rowscale->data_ptr<float>();
    if (coef.has_value() && coef->defined()) {
      TORCH_CHECK(targets.has_value() && wtab.has_value(), "rms_bwd: the exact target form needs targets and w");
      check_rows(*coef, M, 1, at::kFloat, "coef");
      check_rows(*targets, M, 1, at::kInt, "targets");
      TORCH_CHECK(wtab->scalar_type() == at::kFloat && wtab->is_contiguous() && wtab->dim() == 2 &&
                      wtab->size(1) == D, "rms_bwd: w fp32 [V, D]");
      hg.coef = coef->data_ptr<float>();
      hg.targets = targets->data_ptr<int>();
      hg.w = wtab->data_ptr<float>();
      hg.V = (int)wtab->size(0);
    }
  }
  const float* xp = x.data_ptr<float>();
  const float* rp = rstd.data_ptr<float>();
  if (dy.scalar_type() == at::kFloat) {
    if (head)
      rms_bwd_kernel<float, true><<<rows_grid(M), 32 * kWarps, 0, st>>>(xp, rp, dy.data_ptr<float>(), dr, o, ob,
                                                                      (int)M, (int)D, hg);
    else
      rms_bwd_kernel<float, false><<<rows_grid(M), 32 * kWarps, 0, st>>>(xp, rp, dy.data_ptr<float>(), dr, o, ob,
                                                                       (int)M, (int)D, hg);
  } else {
    TORCH_CHECK(!head, "rms_bwd: the head form takes an fp32 dy");
    rms_bwd_kernel<__nv_bfloat16, false><<<rows_grid(M), 32 * kWarps, 0, st>>>(
        xp, rp, reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), dr, o, ob, (int)M, (int)D, hg);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ladder_bwd(const torch::Tensor& x, const torch::Tensor& x0, const torch::Tensor& lam_r,
                const torch::Tensor& lam_0, int64_t layer, const torch::Tensor& rstd, const torch::Tensor& dxn,
                const torch::Tensor& dres, c10::optional<torch::Tensor> dgate_in, torch::Tensor& dx,
                torch::Tensor& dx0_acc, torch::Tensor& dlam_r, torch::Tensor& dlam_0, bool first_layer,
                c10::optional<torch::Tensor> dx_b) {
  const int64_t D = x.size(-1), M = x.numel() / D;
  __nv_bfloat16* dxb = dx_b.has_value() && dx_b->defined() ? reinterpret_cast<__nv_bfloat16*>(dx_b->data_ptr()) : nullptr;
  TORCH_CHECK(!dxb || (dx_b->scalar_type() == at::kBFloat16 && dx_b->is_contiguous()), "ladder_bwd: dx_b bf16");
  c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const float* dgi = dgate_in.has_value() ? dgate_in->data_ptr<float>() : nullptr;
  const int grid = std::min(rows_grid(M), 4 * 148);
  if (dxn.scalar_type() == at::kFloat)
    ladder_bwd_kernel<float><<<grid, 32 * kWarps, 0, st>>>(
        x.data_ptr<float>(), x0.data_ptr<float>(), lam_r.data_ptr<float>(), lam_0.data_ptr<float>(), (int)layer,
        rstd.data_ptr<float>(), dxn.data_ptr<float>(), dres.data_ptr<float>(), dgi, dx.data_ptr<float>(),
        dx0_acc.data_ptr<float>(), dlam_r.data_ptr<float>(), dlam_0.data_ptr<float>(), (int)M, (int)D, first_layer,
        dxb);
  else
    ladder_bwd_kernel<__nv_bfloat16><<<grid, 32 * kWarps, 0, st>>>(
        x.data_ptr<float>(), x0.data_ptr<float>(), lam_r.data_ptr<float>(), lam_0.data_ptr<float>(), (int)layer,
        rstd.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(dxn.data_ptr()), dres.data_ptr<float>(), dgi,
        dx.data_ptr<float>(), dx0_acc.data_ptr<float>(), dlam_r.data_ptr<float>(), dlam_0.data_ptr<float>(), (int)M,
        (int)D, first_layer, dxb);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_bwd(const torch::Tensor& idx, const torch::Tensor& wte, const torch::Tensor& rstd, const torch::Tensor& dx0,
               torch::Tensor& dwte) {
  const int64_t M = idx.numel(), D = wte.size(1);
  c10::cuda::CUDAGuard g(wte.device());
  embed_bwd_kernel<<<rows_grid(M), 32 * kWarps, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int>(), wte.data_ptr<float>(), rstd.data_ptr<float>(), dx0.data_ptr<float>(),
      dwte.data_ptr<float>(), (int)M, (int)D, (int)wte.size(0), status_ptr(wte.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cast_bf16(const torch::Tensor& x, torch::Tensor& y) {
  TORCH_CHECK(x.numel() % 4 == 0 && x.is_contiguous() && y.is_contiguous(), "cast_bf16: contiguous, numel%4");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t n4 = x.numel() / 4;
  const int grid = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 16);
  cast_bf16_kernel<<<std::max(grid, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n4);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br
