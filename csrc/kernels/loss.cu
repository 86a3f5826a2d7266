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
#include "status.h"

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
                                                       float* __restrict__ nats, float* __restrict__ loss_sum,
                                                       int* status) {
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
    int t = targets[row];
    if (t != -1 && !index_ok(t, V, status)) t = -1;  // an id outside the vocabulary is ignored and reported
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
    const int t = targets[row] < V ? targets[row] : -1;
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

// Two forms for the target column: with `g` (the patch form the engine uses) G[m, t] = cf / rowscale in
// bf16, so both backward GEMMs include it and no scatter is needed; with `dw` (the exact fp32 form) the
// gradient is scattered into dW here and added to dx by rms_bwd's head form.
// Finishes the cross-entropy of the fused lm_head epilogue (EPI_SOFTCAP_CE in gemm.cu), whose GEMM wrote
// per (256-column tile half, row) partial sums of e_j = exp(z_j - cap), the target's softcapped logit z_t and
// G = e (1 - (z/cap)^2) with G_t = 0. Per row, with S = sum_j e_j:
//   lse = cap + log S, p_t = exp(z_t - lse), nats = -log(p_t + 1e-10)      (the reference's eps form)
//   dz_j = r (p_j - [j == t]) c'_j, r = scale p_t / (p_t + 1e-10), c' = 1 - (z/cap)^2
//        = rowscale * G_j + [j == t] coef,  rowscale = r / S,  coef = r (p_t - 1) c'_t
// so the backward consumes G with rowscale folded into its other operand and the target column added
// exactly in fp32: dx = rowscale (G W) + coef W[t] (rms_bwd's head form), dW = G^T (rowscale x) plus
// the scatter dW[t] += coef x done here, and xs = bf16(rowscale x) is written for the dW GEMM.
// Rows whose target is -1 are masked (no loss, no gradient, nats 0); any other target outside [0, V) is
// masked the same way and reported as kErrBadIndex.
// Block: 256 rows. Phase 1 is one thread per row (coalesced [tile][row] partials); phase 2 one warp per
// row for the 16-byte vector work on x.
constexpr int kFinRows = 256;

__global__ void __launch_bounds__(kFinRows) ce_finalize_kernel(
    const float* __restrict__ partial, int n_tiles, const float* __restrict__ zt, const int* __restrict__ targets,
    int M, int V, float cap, float scale, float* __restrict__ nats, float* __restrict__ loss_sum,
    float* __restrict__ rowscale, float* __restrict__ coef, const __nv_bfloat16* __restrict__ x,
    __nv_bfloat16* __restrict__ xs, float* __restrict__ dw, int D, __nv_bfloat16* __restrict__ g, int64_t ldg,
    int* status) {
  __shared__ float s_rs[kFinRows], s_cf[kFinRows], s_red[kFinRows / 32];
  __shared__ int s_t[kFinRows];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = blockIdx.x * kFinRows; base < M; base += gridDim.x * kFinRows) {
    const int m = base + threadIdx.x;
    float contrib = 0.f;
    if (m < M) {
      float S = 0.f;
      for (int n = 0; n < n_tiles; ++n) S += __ldg(partial + (int64_t)n * M + m);
      const int t = __ldg(targets + m);
      const bool valid = t == -1 ? false : index_ok(t, V, status);  // -1: ignored position
      const float z = valid ? __ldg(zt + m) : 0.f;
      const float pt = __expf(z - cap - __logf(S));
      const float nll = -__logf(pt + 1e-10f);
      if (nats) nats[m] = valid ? nll : 0.f;
      contrib = valid ? nll * scale : 0.f;
      const float r = valid ? scale * (pt / (pt + 1e-10f)) : 0.f;
      const float zc = z / cap;
      const float rs = r / S, cf = r * (pt - 1.f) * (1.f - zc * zc);
      if (rowscale) rowscale[m] = rs;
      if (coef) coef[m] = cf;
      // patch form: the target column's gradient goes into G itself (scaled so that rowscale * G gives it)
      if (g && valid && rs > 0.f) g[(int64_t)m * ldg + t] = __float2bfloat16(cf / rs);
      s_rs[threadIdx.x] = rs;
      s_cf[threadIdx.x] = cf;
      s_t[threadIdx.x] = valid ? t : -1;
    }
    if (loss_sum) {
      const float w = warp_sum(contrib);
      if (lane == 0) s_red[warp] = w;
    }
    __syncthreads();
    if (loss_sum && threadIdx.x == 0) {
      float tot = 0.f;
      for (int i = 0; i < kFinRows / 32; ++i) tot += s_red[i];
      atomicAdd(loss_sum, tot);
    }
    if (x) {
      for (int i = warp; i < kFinRows && base + i < M; i += kFinRows / 32) {
        const int64_t row = base + i;
        const float rs = s_rs[i], cf = s_cf[i];
        const int t = s_t[i];
        for (int c = lane * 8; c < D; c += 256) {
          const uint4 u = *reinterpret_cast<const uint4*>(x + row * D + c);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          float v[8];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16(w[k]);
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
          }
          if (xs)
            *reinterpret_cast<uint4*>(xs + row * D + c) =
                make_uint4(pack_bf16(rs * v[0], rs * v[1]), pack_bf16(rs * v[2], rs * v[3]),
                           pack_bf16(rs * v[4], rs * v[5]), pack_bf16(rs * v[6], rs * v[7]));
          if (dw && t >= 0) {
            float* d = dw + (int64_t)t * D + c;
            red_add_v4_f32(d, cf * v[0], cf * v[1], cf * v[2], cf * v[3]);
            red_add_v4_f32(d + 4, cf * v[4], cf * v[5], cf * v[6], cf * v[7]);
          }
        }
      }
    }
    __syncthreads();  // the shared row data is rewritten by the next row block
  }
}

}  // namespace

void ce_finalize(const torch::Tensor& partial, const torch::Tensor& zt, const torch::Tensor& targets, int64_t V,
                 double cap, double scale, c10::optional<torch::Tensor> nats, c10::optional<torch::Tensor> loss_sum,
                 c10::optional<torch::Tensor> rowscale, c10::optional<torch::Tensor> coef,
                 c10::optional<torch::Tensor> x, c10::optional<torch::Tensor> xs, c10::optional<torch::Tensor> dw,
                 c10::optional<torch::Tensor> g) {
  const int64_t M = targets.numel();
  const int64_t n_tiles = 2 * ((V + 255) / 256);  // two partial rows per 256-column tile
  TORCH_CHECK(targets.scalar_type() == at::kInt && targets.is_contiguous(), "ce_finalize: int32 targets");
  TORCH_CHECK(partial.scalar_type() == at::kFloat && partial.is_contiguous() && partial.numel() >= n_tiles * M,
              "ce_finalize: partial fp32 [2 ceil(V/256), M]");
  TORCH_CHECK(zt.scalar_type() == at::kFloat && zt.numel() >= M, "ce_finalize: zt fp32 [M]");
  auto f32 = [&](const c10::optional<torch::Tensor>& t, const char* name) -> float* {
    if (!t.has_value() || !t->defined()) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() >= M, "ce_finalize: ", name);
    return t->data_ptr<float>();
  };
  int64_t D = 0;
  const __nv_bfloat16* xp = nullptr;
  __nv_bfloat16* xsp = nullptr;
  float* dwp = nullptr;
  if (x.has_value() && x->defined()) {
    TORCH_CHECK(x->scalar_type() == at::kBFloat16 && x->is_contiguous() && x->dim() == 2 && x->size(0) == M,
                "ce_finalize: x bf16 [M, D]");
    D = x->size(1);
    TORCH_CHECK(D % 8 == 0, "ce_finalize: D % 8");
    xp = reinterpret_cast<const __nv_bfloat16*>(x->data_ptr());
    if (xs.has_value() && xs->defined()) {
      TORCH_CHECK(xs->scalar_type() == at::kBFloat16 && xs->is_contiguous() && xs->numel() == M * D, "ce_finalize: xs");
      xsp = reinterpret_cast<__nv_bfloat16*>(xs->data_ptr());
    }
    if (dw.has_value() && dw->defined()) {
      TORCH_CHECK(dw->scalar_type() == at::kFloat && dw->is_contiguous() && dw->numel() == V * D, "ce_finalize: dw");
      dwp = dw->data_ptr<float>();
    }
  }
  __nv_bfloat16* gp = nullptr;
  int64_t ldg = 0;
  if (g.has_value() && g->defined()) {
    TORCH_CHECK(g->scalar_type() == at::kBFloat16 && g->dim() == 2 && g->size(0) == M && g->size(1) == V &&
                    g->stride(1) == 1, "ce_finalize: g bf16 [M, V] with contiguous rows");
    TORCH_CHECK(rowscale.has_value() && rowscale->defined(), "ce_finalize: the patch form needs rowscale");
    gp = reinterpret_cast<__nv_bfloat16*>(g->data_ptr());
    ldg = g->stride(0);
  }
  float* ls = nullptr;
  if (loss_sum.has_value() && loss_sum->defined()) {
    TORCH_CHECK(loss_sum->scalar_type() == at::kFloat, "ce_finalize: loss_sum fp32");
    ls = loss_sum->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(targets.device());
  int dev = targets.device().index(), sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t blocks = std::min<int64_t>((M + kFinRows - 1) / kFinRows, (int64_t)sms * 8);
  ce_finalize_kernel<<<(unsigned)std::max<int64_t>(blocks, 1), kFinRows, 0, at::cuda::getCurrentCUDAStream()>>>(
      partial.data_ptr<float>(), (int)n_tiles, zt.data_ptr<float>(), targets.data_ptr<int>(), (int)M, (int)V,
      (float)cap, (float)scale, f32(nats, "nats"), ls, f32(rowscale, "rowscale"), f32(coef, "coef"), xp, xsp, dwp,
      (int)D, gp, ldg, status_ptr(targets.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

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
                                                       (float)cap, (float)scale, n, ls,
                                                       status_ptr(logits.device().index()));
  else
    ce_kernel<false><<<(unsigned)M, kThreads, 0, st>>>(L, logits.stride(0), targets.data_ptr<int>(), (int)V,
                                                        (float)cap, (float)scale, n, ls,
                                                       status_ptr(logits.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br
