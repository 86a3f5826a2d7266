// Fused optimizer kernels (src/train/muon.ts).
//
//   adamw_multi        one launch over all AdamW tensors of a step (muon.ts:60-96): decoupled decay,
//                      moment EMAs, bias-corrected update, optional bf16 shadow write.
//   muon_momentum      Nesterov momentum for a stack of equally-shaped matrices (muon.ts:151-152):
//                      mom = mu*mom + (1-mu)*g, g' = (1-mu)*g + mu*mom, and sum(g'^2) per matrix.
//   muon_normalize     X = bf16(g' / (||g'||_F * 1.02 + 1e-6)) (muon.ts:108-109), packed [S, r, c].
//   normuon_stats      v_mean over the reduction dim (cols when r >= c, else rows), second-moment
//                      EMA update (beta2) and the two per-matrix sums of the NorMuon rescale
//                      (muon.ts:158-181).
//   muon_apply         p -= lr * (X * final_scale + wd * p * [g*p >= 0]) (muon.ts:183-194), fp32
//                      master plus bf16 shadow.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace br {
namespace {

constexpr int kMaxT = 32;

struct AdamTensor {
  float* p;
  const float* g;
  float* m;
  float* v;
  __nv_bfloat16* shadow;
  int64_t n;
  float lr, b1, b2, bias1, bias2, eps, wd;
  int64_t block0;  // first block index of this tensor
};

struct AdamBatch {
  AdamTensor t[kMaxT];
  int count;
  const int* skip;  // nonzero: leave every tensor unchanged (the step's update is skipped on the device)
};

constexpr int kAdamPerBlock = 256 * 8;

__global__ void adamw_kernel(const __grid_constant__ AdamBatch b) {
  if (b.skip && *b.skip) return;
  int ti = 0;
  while (ti + 1 < b.count && blockIdx.x >= b.t[ti + 1].block0) ++ti;
  const AdamTensor& T = b.t[ti];
  const int64_t base = (int64_t)(blockIdx.x - T.block0) * kAdamPerBlock;
  const float step = T.lr / T.bias1;
  const float inv_b2 = 1.f / T.bias2;
  for (int k = threadIdx.x; k < kAdamPerBlock; k += blockDim.x) {
    const int64_t i = base + k;
    if (i >= T.n) break;
    const float g = T.g[i];
    float p = T.p[i] * (1.f - T.lr * T.wd);
    const float m = T.b1 * T.m[i] + (1.f - T.b1) * g;
    const float v = T.b2 * T.v[i] + (1.f - T.b2) * g * g;
    p -= step * m / (sqrtf(v * inv_b2) + T.eps);
    T.p[i] = p;
    T.m[i] = m;
    T.v[i] = v;
    if (T.shadow) T.shadow[i] = __float2bfloat16(p);
  }
}

struct MatPtrs {
  const float* g[64];
  float* mom[64];
  float* p[64];
  float* sec[64];
  __nv_bfloat16* shadow[64];
  int64_t shadow_ld[64];
};

// Block sum in a fixed order (warp tree, then the warps' sums in index order): the same inputs give the same
// bits on every rank, so replicated optimizer steps keep replicas identical (float atomics would not).
__device__ __forceinline__ float block_sum_fixed(float v) {
  __shared__ float warps[32];
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) warps[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += warps[w];
  __syncthreads();
  return t;  // valid in thread 0
}

// grid: (chunks, S). part[s * chunks + chunk] = this block's sum(g'^2).
__global__ void muon_momentum_kernel(const __grid_constant__ MatPtrs P, int64_t n, float mu, float* __restrict__ part,
                                     const int* skip) {
  if (skip && *skip) return;  // momentum unchanged; the NS iteration then runs on stale data, never applied
  const int s = blockIdx.y;
  const float* g = P.g[s];
  float* mom = P.mom[s];
  float acc = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i];
    const float mi = mu * mom[i] + (1.f - mu) * gi;
    mom[i] = mi;
    const float gp = (1.f - mu) * gi + mu * mi;
    acc += gp * gp;
  }
  acc = block_sum_fixed(acc);
  if (threadIdx.x == 0) part[(int64_t)s * gridDim.x + blockIdx.x] = acc;
}

// Every block sums the partials of its matrix in chunk order (the same result in every block and on
// every rank); block 0 also stores the total in ss[s].
__global__ void muon_normalize_kernel(const __grid_constant__ MatPtrs P, int64_t n, float mu,
                                      const float* __restrict__ part, float* __restrict__ ss,
                                      __nv_bfloat16* __restrict__ X) {
  const int s = blockIdx.y;
  const float* g = P.g[s];
  const float* mom = P.mom[s];
  __shared__ float tot;
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int c = 0; c < (int)gridDim.x; ++c) t += part[(int64_t)s * gridDim.x + c];
    tot = t;
    if (blockIdx.x == 0) ss[s] = t;
  }
  __syncthreads();
  const float inv = 1.f / (sqrtf(tot) * 1.02f + 1e-6f);
  __nv_bfloat16* x = X + (int64_t)s * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = __float2bfloat16(((1.f - mu) * g[i] + mu * mom[i]) * inv);
}

// One thread per reduction line (row when r >= c, column otherwise); grid (ceil(lines/256), S).
// Block partials: sums[2 * (s * nblk + blk)] = sum(v_mean * red), [.. + 1] = sum(v_mean * red * step^2).
__global__ void normuon_stats_kernel(const __nv_bfloat16* __restrict__ X, const __grid_constant__ MatPtrs P, int r,
                                     int c, float beta2, float* __restrict__ vmean_out, float* __restrict__ sums,
                                     const int* skip) {
  if (skip && *skip) return;
  const int s = blockIdx.y;
  const bool rows_major = r >= c;
  const int lines = rows_major ? r : c;
  const int red = rows_major ? c : r;
  const int line = blockIdx.x * blockDim.x + threadIdx.x;
  float a = 0.f, b = 0.f;
  if (line < lines) {
    const __nv_bfloat16* x = X + (int64_t)s * r * c;
    float acc = 0.f;
    if (rows_major) {
      const __nv_bfloat16* row = x + (int64_t)line * c;
      for (int j = 0; j < c; ++j) {
        const float v = __bfloat162float(row[j]);
        acc += v * v;
      }
    } else {
      for (int i = 0; i < r; ++i) {
        const float v = __bfloat162float(x[(int64_t)i * c + line]);
        acc += v * v;
      }
    }
    const float vm = acc / red;
    float* sec = P.sec[s];
    const float ns = sec[line] * beta2 + vm * (1.f - beta2);
    sec[line] = ns;
    const float st = rsqrtf(ns + 1e-10f);
    vmean_out[(int64_t)s * lines + line] = st;  // step size per line
    a = vm * red;
    b = vm * red * st * st;
  }
  a = block_sum_fixed(a);
  b = block_sum_fixed(b);
  if (threadIdx.x == 0) {
    const int64_t o = 2 * ((int64_t)s * gridDim.x + blockIdx.x);
    sums[o] = a;
    sums[o + 1] = b;
  }
}

__global__ void muon_apply_kernel(const __nv_bfloat16* __restrict__ X, const __grid_constant__ MatPtrs P, int r, int c,
                                  const float* __restrict__ step_sz, const float* __restrict__ sums, int nblk,
                                  float lr, float wd, const int* skip) {
  if (skip && *skip) return;
  const int s = blockIdx.y;
  const bool rows_major = r >= c;
  const int lines = rows_major ? r : c;
  __shared__ float ratio_s;
  if (threadIdx.x == 0) {  // the stats kernel's block partials, in block order
    float a = 0.f, b = 0.f;
    for (int k = 0; k < nblk; ++k) {
      a += sums[2 * ((int64_t)s * nblk + k)];
      b += sums[2 * ((int64_t)s * nblk + k) + 1];
    }
    ratio_s = sqrtf(a) / (sqrtf(b) + 1e-10f);
  }
  __syncthreads();
  const float ratio = ratio_s;
  const int64_t n = (int64_t)r * c;
  const __nv_bfloat16* x = X + (int64_t)s * n;
  float* p = P.p[s];
  const float* g = P.g[s];
  __nv_bfloat16* sh = P.shadow[s];
  const int64_t sld = P.shadow_ld[s];
  const float* st = step_sz + (int64_t)s * lines;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / c), col = (int)(i % c);
    const float fs = st[rows_major ? row : col] * ratio;
    const float pi = p[i];
    const float mask = g[i] * pi >= 0.f ? 1.f : 0.f;
    const float np = pi - lr * (__bfloat162float(x[i]) * fs + wd * pi * mask);
    p[i] = np;
    if (sh) sh[(int64_t)row * sld + col] = __float2bfloat16(np);
  }
}

int sms() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

MatPtrs make_ptrs(const std::vector<torch::Tensor>& g, const std::vector<torch::Tensor>& mom,
                  const std::vector<torch::Tensor>& p, const std::vector<torch::Tensor>& sec,
                  const std::vector<torch::Tensor>& shadow) {
  MatPtrs P{};
  TORCH_CHECK(g.size() <= 64, "muon: at most 64 matrices per stack");
  for (size_t i = 0; i < g.size(); ++i) {
    P.g[i] = g[i].data_ptr<float>();
    if (!mom.empty()) P.mom[i] = mom[i].data_ptr<float>();
    if (!p.empty()) P.p[i] = p[i].data_ptr<float>();
    if (!sec.empty()) P.sec[i] = sec[i].data_ptr<float>();
    if (!shadow.empty() && shadow[i].defined()) {
      P.shadow[i] = reinterpret_cast<__nv_bfloat16*>(shadow[i].data_ptr());
      P.shadow_ld[i] = shadow[i].stride(0);
    }
  }
  return P;
}

}  // namespace

// Scratch sizes (floats) of the two Muon entry points, for callers that allocate it once.
int64_t muon_prepare_scratch(int64_t S, int64_t n) {
  const int64_t chunks = std::max<int64_t>(1, std::min<int64_t>((n + 1023) / 1024, 4 * sms() / std::max<int64_t>(S, 1) + 1));
  return S + S * chunks;
}
int64_t muon_finish_scratch(int64_t S, int64_t r, int64_t c) {
  const int64_t lines = r >= c ? r : c;
  return 2 * S * ((lines + 255) / 256) + S * lines;
}

void adamw_multi(const std::vector<torch::Tensor>& params, const std::vector<torch::Tensor>& grads,
                 const std::vector<torch::Tensor>& ms, const std::vector<torch::Tensor>& vs,
                 const std::vector<torch::Tensor>& shadows, const std::vector<double>& hyper,
                 c10::optional<torch::Tensor> skip) {
  // hyper: per tensor [lr, b1, b2, bias1, bias2, eps, wd]; skip: optional int32 [1] device word
  const size_t n = params.size();
  TORCH_CHECK(n <= (size_t)kMaxT && hyper.size() == 7 * n, "adamw_multi: bad arguments");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(params[0].device());
  AdamBatch b{};
  int64_t blocks = 0;
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(params[i].is_contiguous() && grads[i].is_contiguous(), "adamw_multi: contiguous tensors");
    AdamTensor& t = b.t[i];
    t.p = params[i].data_ptr<float>();
    t.g = grads[i].data_ptr<float>();
    t.m = ms[i].data_ptr<float>();
    t.v = vs[i].data_ptr<float>();
    t.shadow = shadows[i].defined() ? reinterpret_cast<__nv_bfloat16*>(shadows[i].data_ptr()) : nullptr;
    t.n = params[i].numel();
    t.lr = (float)hyper[7 * i];
    t.b1 = (float)hyper[7 * i + 1];
    t.b2 = (float)hyper[7 * i + 2];
    t.bias1 = (float)hyper[7 * i + 3];
    t.bias2 = (float)hyper[7 * i + 4];
    t.eps = (float)hyper[7 * i + 5];
    t.wd = (float)hyper[7 * i + 6];
    t.block0 = blocks;
    blocks += (t.n + kAdamPerBlock - 1) / kAdamPerBlock;
  }
  b.count = (int)n;
  b.skip = skip.has_value() && skip->defined() ? skip->data_ptr<int>() : nullptr;
  adamw_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(b);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Returns X (bf16 [S, r, c]) normalised for Newton-Schulz; updates momentum buffers in place.
void muon_prepare(const std::vector<torch::Tensor>& grads, const std::vector<torch::Tensor>& moms, double mu,
                  torch::Tensor& X, torch::Tensor& ss, c10::optional<torch::Tensor> skip) {
  const int* sk = skip.has_value() && skip->defined() ? skip->data_ptr<int>() : nullptr;
  const int S = (int)grads.size();
  const int64_t n = grads[0].numel();
  c10::cuda::CUDAGuard guard(grads[0].device());
  auto st = at::cuda::getCurrentCUDAStream();
  MatPtrs P = make_ptrs(grads, moms, {}, {}, {});
  const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 1023) / 1024, 4 * sms() / std::max(S, 1) + 1));
  // ss: [S] totals followed by [S, chunks] block partials
  TORCH_CHECK(ss.scalar_type() == at::kFloat && ss.numel() >= muon_prepare_scratch(S, n),
              "muon_prepare: ss needs muon_prepare_scratch(S, n) floats");
  float* part = ss.data_ptr<float>() + S;
  dim3 grid(chunks, S);
  muon_momentum_kernel<<<grid, 256, 0, st>>>(P, n, (float)mu, part, sk);
  muon_normalize_kernel<<<grid, 256, 0, st>>>(P, n, (float)mu, part, ss.data_ptr<float>(),
                                              reinterpret_cast<__nv_bfloat16*>(X.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void muon_finish(const torch::Tensor& X, const std::vector<torch::Tensor>& grads,
                 const std::vector<torch::Tensor>& params, const std::vector<torch::Tensor>& secs,
                 const std::vector<torch::Tensor>& shadows, int64_t r, int64_t c, double beta2, double lr, double wd,
                 torch::Tensor& work, c10::optional<torch::Tensor> skip) {
  const int* sk = skip.has_value() && skip->defined() ? skip->data_ptr<int>() : nullptr;
  const int S = (int)grads.size();
  c10::cuda::CUDAGuard guard(X.device());
  auto st = at::cuda::getCurrentCUDAStream();
  MatPtrs P = make_ptrs(grads, {}, params, secs, shadows);
  const int lines = (int)(r >= c ? r : c);
  const int nblk = (lines + 255) / 256;
  // work: [2 * S * nblk] block partial sums, then [S * lines] per-line step sizes
  TORCH_CHECK(work.numel() >= muon_finish_scratch(S, r, c), "muon_finish: work needs muon_finish_scratch(S, r, c) floats");
  float* sums = work.data_ptr<float>();
  float* step_sz = sums + 2 * (int64_t)S * nblk;
  normuon_stats_kernel<<<dim3(nblk, S), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()), P, (int)r, (int)c, (float)beta2, step_sz, sums, sk);
  const int64_t n = r * c;
  const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 1023) / 1024, 4 * sms() / std::max(S, 1) + 1));
  muon_apply_kernel<<<dim3(chunks, S), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()), P, (int)r,
                                                     (int)c, step_sz, sums, nblk, (float)lr, (float)wd, sk);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br
