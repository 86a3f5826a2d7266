// Monte-Carlo Sharpe distribution of a strategy, one GBM price path per thread (the strategy swarm's
// inner loop, swarm.html:214-236 in the reference, which runs it in plain JS: 50,000 paths x 252 steps
// per variant).
//
// Path p: price_t = price_{t-1} exp(drift + diffusion z_t), t = 1 .. steps-1, z_t ~ N(0, 1). The
// path's simple returns r_t = exp(drift + diffusion z_t) - 1 are scored like the reference's
// computeSharpe (swarm.html:143-151): the series is shifted by one (0, r_1 .. r_{n-1}, the last return
// dropped), mean and population variance over those n values, Sharpe = mean / std * sqrt(annual), -9
// when std <= 1e-9 or n < 10.
//
// Normals: a counter-based generator (SplitMix64 finaliser over (seed, path, step)), two 24-bit
// uniforms in (0, 1), Box-Muller (cos branch, as the reference's randn). Each thread keeps a running
// sum and sum of squares (fp64 for the variance), so a path needs no storage.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

namespace br {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256) mc_sharpe_kernel(float* __restrict__ out, int n_paths, int steps,
                                                        double drift, double diffusion, double annual,
                                                        uint64_t seed) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n_paths) return;
  const uint64_t base = mix64(seed ^ (0xd1b54a32d192ed03ull * (uint64_t)(p + 1)));
  // shifted series: x_0 = 0, x_t = r_t for t = 1 .. n-1 where n = steps - 1 returns exist
  const int n = steps - 1;
  double s = 0.0, ss = 0.0;
  for (int t = 1; t < n; ++t) {
    const uint64_t u = mix64(base + (uint64_t)t);
    const float u1 = ((float)(u >> 40) + 0.5f) * (1.f / 16777216.f);           // (0, 1)
    const float u2 = ((float)((u >> 16) & 0xffffffull) + 0.5f) * (1.f / 16777216.f);
    const float z = sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    const double r = exp(drift + diffusion * (double)z) - 1.0;
    s += r;
    ss += r * r;
  }
  if (n < 10) {
    out[p] = -9.f;
    return;
  }
  const double m = s / n;
  const double v = fmax(ss / n - m * m, 0.0);
  const double sd = sqrt(v);
  out[p] = sd > 1e-9 ? (float)(m / sd * sqrt(annual)) : -9.f;
}

}  // namespace

// Sharpe ratios of n_paths simulated GBM paths of `steps` prices with annualised drift mu and volatility
// sigma (the moments of the strategy's daily returns), as fp32 [n_paths] on `device`.
torch::Tensor mc_sharpe(int64_t n_paths, int64_t steps, double mu, double sigma, double annual, int64_t seed,
                        int64_t device) {
  TORCH_CHECK(n_paths > 0 && steps > 1, "mc_sharpe: n_paths > 0, steps > 1");
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  auto out = torch::empty({n_paths}, torch::dtype(torch::kFloat32).device(torch::kCUDA, (c10::DeviceIndex)device));
  const double dt = 1.0 / annual;
  const double drift = (mu - 0.5 * sigma * sigma) * dt;
  const double diffusion = sigma * std::sqrt(dt);
  mc_sharpe_kernel<<<(unsigned)((n_paths + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<float>(), (int)n_paths, (int)steps, drift, diffusion, annual, (uint64_t)seed);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace br
