// Persistent warp-specialised tcgen05 GEMM for sm_100a: C[b] = epilogue(A[b] . B[b]^T).
//
//   A: logical [M, K], either K-major (stored [M, K]) or MN-major (stored [K, M]).
//   B: logical [N, K], either K-major (stored [N, K]) or MN-major (stored [K, N]).
//   bf16 operands, fp32 accumulation in TMEM, 128 x BN x 64 tiles (BN = 128 or 256).
//
// Roles (192 threads, one CTA per SM, grid = min(work units, SMs)):
//   warp 0  one elected lane issues TMA loads (128-byte swizzle, no multicast) into a
//           STAGES-deep ring of shared-memory stages guarded by full/empty mbarriers;
//   warp 1  allocates TMEM (two BN-column fp32 accumulators) and one elected lane issues
//           tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit;
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM lanes 32*(w%4)..),
//           applies the fused epilogue and stores; the accumulator is released to the MMA warp
//           through tmem_empty so the next tile's main loop overlaps this epilogue.
// Work units are (k-split, n-tile, m-tile, batch) with n fastest so CTAs running at the same time
// share A rows through L2. With k_splits > 1 each unit accumulates its fp32 partial into C with
// vector reductions (used for weight gradients, whose reduction dimension is the token count).
//
// All mbarrier waits are bounded (2 s); on timeout the kernel records a status code, drains its
// in-flight TMA loads and MMAs, frees TMEM and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "status.h"

namespace br {

enum GemmEpi : int {
  EPI_BF16 = 0,        // C(bf16) = alpha*acc + beta*aux(bf16, optional)
  EPI_F32 = 1,         // C(f32)  = alpha*acc + beta*aux(f32, optional; may alias C)
  EPI_RELU2 = 2,       // C(bf16) = relu(alpha*acc)^2
  EPI_RELU2_BWD = 3,   // C(bf16) = alpha*acc * 2*sqrt(aux(bf16))   (d/du of relu(u)^2 given h = relu(u)^2)
  EPI_ATOMIC_F32 = 4,  // C(f32) += alpha*acc
  EPI_SOFTCAP = 5,     // C(bf16) = beta*tanh(alpha*acc)             (alpha = 1/cap, beta = cap)
};

struct GemmParams {
  int M, N, K, batch;
  int k_splits, kb_per_split;
  int m_tiles, n_tiles, k_blocks;
  void* C;
  int64_t ldc, bsc;
  const void* aux;
  int64_t ld_aux, bs_aux;
  float alpha, beta;
  int* status;
};

constexpr int BM = 128;
constexpr int BK = 64;
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void decode_unit(const GemmParams& p, int u, int& m, int& n, int& b, int& kb0, int& kb1) {
  int s = u % p.k_splits;
  int r = u / p.k_splits;
  n = r % p.n_tiles;
  r /= p.n_tiles;
  m = r % p.m_tiles;
  b = r / p.m_tiles;
  kb0 = s * p.kb_per_split;
  kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int b, int row, int col0, uint32_t (&r)[32]) {
  if (row >= p.M) return;
  const bool full = col0 + 32 <= p.N;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
  if constexpr (EPI == EPI_BF16 || EPI == EPI_RELU2 || EPI == EPI_RELU2_BWD || EPI == EPI_SOFTCAP) {
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C) + (int64_t)b * p.bsc + (int64_t)row * p.ldc + col0;
    const __nv_bfloat16* X = p.aux ? reinterpret_cast<const __nv_bfloat16*>(p.aux) + (int64_t)b * p.bs_aux +
                                         (int64_t)row * p.ld_aux + col0
                                   : nullptr;
    if (full) {
      if constexpr (EPI == EPI_BF16 || EPI == EPI_RELU2_BWD) {
        if (X) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 xv = *reinterpret_cast<const uint4*>(X + q * 8);
            uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float2 f = unpack_bf16(xs[j]);
              if constexpr (EPI == EPI_BF16) {
                v[q * 8 + 2 * j] += p.beta * f.x;
                v[q * 8 + 2 * j + 1] += p.beta * f.y;
              } else {
                v[q * 8 + 2 * j] *= 2.f * sqrtf(fmaxf(f.x, 0.f));
                v[q * 8 + 2 * j + 1] *= 2.f * sqrtf(fmaxf(f.y, 0.f));
              }
            }
          }
        }
      }
      if constexpr (EPI == EPI_RELU2) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float t = fmaxf(v[i], 0.f);
          v[i] = t * t;
        }
      }
      if constexpr (EPI == EPI_SOFTCAP) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = p.beta * tanhf(v[i]);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 o;
        o.x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
        *reinterpret_cast<uint4*>(C + q * 8) = o;
      }
    } else {
      for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
        float x = v[i];
        if constexpr (EPI == EPI_BF16) {
          if (X) x += p.beta * __bfloat162float(X[i]);
        } else if constexpr (EPI == EPI_RELU2_BWD) {
          x *= 2.f * sqrtf(fmaxf(__bfloat162float(X[i]), 0.f));
        } else if constexpr (EPI == EPI_RELU2) {
          x = fmaxf(x, 0.f);
          x = x * x;
        } else {
          x = p.beta * tanhf(x);
        }
        C[i] = __float2bfloat16(x);
      }
    }
  } else {  // fp32 outputs
    float* C = reinterpret_cast<float*>(p.C) + (int64_t)b * p.bsc + (int64_t)row * p.ldc + col0;
    if constexpr (EPI == EPI_ATOMIC_F32) {
      if (full) {
#pragma unroll
        for (int q = 0; q < 8; ++q) red_add_v4_f32(C + q * 4, v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
      } else {
        for (int i = 0; i < 32 && col0 + i < p.N; ++i) atomicAdd(C + i, v[i]);
      }
    } else {
      const float* X = p.aux ? reinterpret_cast<const float*>(p.aux) + (int64_t)b * p.bs_aux +
                                   (int64_t)row * p.ld_aux + col0
                             : nullptr;
      if (full) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 o = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
          if (X) {
            float4 x = *reinterpret_cast<const float4*>(X + q * 4);
            o.x += p.beta * x.x;
            o.y += p.beta * x.y;
            o.z += p.beta * x.z;
            o.w += p.beta * x.w;
          }
          *reinterpret_cast<float4*>(C + q * 4) = o;
        }
      } else {
        for (int i = 0; i < 32 && col0 + i < p.N; ++i) C[i] = v[i] + (X ? p.beta * X[i] : 0.f);
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint64_t* drain_bar = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int total = p.m_tiles * p.n_tiles * p.batch * p.k_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto fail = [&](int code) {
    *abort_flag = 1;
    if (p.status) atomicCAS(p.status, 0, code);
  };

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        int m, n, b, kb0, kb1;
        decode_unit(p, u, m, n, b, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, kWaitBudgetNs, abort_flag)) {
            fail(kErrTimeoutProducer);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          if constexpr (!A_MN) {
            tma_load_3d(&tmA, &full_bar[stage], a_dst, kb * BK, m * BM, b);
          } else {
            tma_load_3d(&tmA, &full_bar[stage], a_dst, m * BM, kb * BK, b);
            tma_load_3d(&tmA, &full_bar[stage], a_dst + 8192, m * BM + 64, kb * BK, b);
          }
          if constexpr (!B_MN) {
            tma_load_3d(&tmB, &full_bar[stage], b_dst, kb * BK, n * BN, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(&tmB, &full_bar[stage], b_dst + j * 8192, n * BN + j * 64, kb * BK, b);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok || *abort_flag) {
        // wait (bounded) for the loads still in flight before the CTA's shared memory goes away
        int n_inflight = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < n_inflight; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(&full_bar[s], ph, 100000000ull, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++local) {
        int m, n, b, kb0, kb1;
        decode_unit(p, u, m, n, b, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, kWaitBudgetNs, abort_flag)) {
          fail(kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kWaitBudgetNs, abort_flag)) {
            fail(kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? umma_desc_sw128(a_base + k * 2048, 8192, 1024)
                                     : umma_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_desc_sw128(b_base + k * 2048, 8192, 1024)
                                     : umma_desc_sw128(b_base + k * 32, 16, 1024);
            umma_bf16_ss(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
      // all MMAs issued by this thread have completed once drain_bar flips
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, 100000000ull, nullptr);
    }
  } else {
    // epilogue warps 2..5
    const int wq = warp & 3;
    const int lane = lane_id();
    int local = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++local) {
      int m, n, b, kb0, kb1;
      decode_unit(p, u, m, n, b, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, kWaitBudgetNs, abort_flag)) {
        fail(kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const int row = m * BM + wq * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait();
        epilogue_chunk<EPI>(p, b, row, n * BN + c * 32, r);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------------- host
namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// 3-D bf16 map over storage [batch][outer][inner] with a 128-byte-swizzled box {64, box_outer, 1}.
CUtensorMap make_map(const void* base, int64_t inner, int64_t outer, int64_t batch, int64_t ld_elems,
                     int64_t bs_elems, int box_outer) {
  CUtensorMap m;
  if (batch == 1 || bs_elems == 0) bs_elems = ld_elems * outer;  // unused for one batch, but must be a valid stride
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld_elems * 2), (cuuint64_t)(bs_elems * 2)};
  cuuint32_t box[3] = {64, (cuuint32_t)box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld_elems * 2) % 16 == 0 && (bs_elems * 2) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

template <int BN, bool AMN, bool BMN, int EPI>
void launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid, cudaStream_t st) {
  auto k = gemm_kernel<BN, AMN, BMN, EPI>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM));
    attr = true;
  }
  k<<<grid, 192, GemmCfg<BN>::SMEM, st>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, bool AMN, bool BMN>
void dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid, cudaStream_t st) {
  switch (epi) {
    case EPI_BF16: return launch_t<BN, AMN, BMN, EPI_BF16>(ta, tb, p, grid, st);
    case EPI_F32: return launch_t<BN, AMN, BMN, EPI_F32>(ta, tb, p, grid, st);
    case EPI_ATOMIC_F32: return launch_t<BN, AMN, BMN, EPI_ATOMIC_F32>(ta, tb, p, grid, st);
    default: break;
  }
  if constexpr (BN == 256) {
    switch (epi) {
      case EPI_RELU2: return launch_t<BN, AMN, BMN, EPI_RELU2>(ta, tb, p, grid, st);
      case EPI_RELU2_BWD: return launch_t<BN, AMN, BMN, EPI_RELU2_BWD>(ta, tb, p, grid, st);
      case EPI_SOFTCAP: return launch_t<BN, AMN, BMN, EPI_SOFTCAP>(ta, tb, p, grid, st);
      default: break;
    }
  }
  TORCH_CHECK(false, "unsupported gemm epilogue ", epi, " for BN=", BN);
}

template <int BN>
void dispatch_major(bool amn, bool bmn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                    int grid, cudaStream_t st) {
  if (!amn && !bmn) return dispatch_epi<BN, false, false>(epi, ta, tb, p, grid, st);
  if (!amn && bmn) return dispatch_epi<BN, false, true>(epi, ta, tb, p, grid, st);
  if (amn && !bmn) return dispatch_epi<BN, true, false>(epi, ta, tb, p, grid, st);
  return dispatch_epi<BN, true, true>(epi, ta, tb, p, grid, st);
}

}  // namespace

// Operands are passed as raw storage with explicit layout:
//   a: storage [batch][M][K] (a_mn=0) or [batch][K][M] (a_mn=1), row stride lda, batch stride bsa
//   b: storage [batch][N][K] (b_mn=0) or [batch][K][N] (b_mn=1), row stride ldb, batch stride bsb
//   c: [batch][M][N] with row stride ldc, batch stride bsc (bf16 or f32 by epilogue)
void gemm_launch(const torch::Tensor& a, bool a_mn, int64_t lda, int64_t bsa, const torch::Tensor& b, bool b_mn,
                 int64_t ldb, int64_t bsb, torch::Tensor& c, int64_t ldc, int64_t bsc, int64_t M, int64_t N,
                 int64_t K, int64_t batch, int64_t epi, c10::optional<torch::Tensor> aux, int64_t ld_aux,
                 int64_t bs_aux, double alpha, double beta, int64_t k_splits, int64_t block_n) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  const bool f32_out = epi == EPI_F32 || epi == EPI_ATOMIC_F32;
  TORCH_CHECK(c.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm: output dtype mismatch");
  TORCH_CHECK(M > 0 && N > 0 && K > 0 && batch > 0, "gemm: empty problem");
  TORCH_CHECK(ldc % 8 == 0, "gemm: ldc must be a multiple of 8");
  c10::cuda::CUDAGuard guard(a.device());
  const int BN = block_n > 0 ? (int)block_n : (N <= 128 ? 128 : 256);
  TORCH_CHECK(BN == 128 || BN == 256, "block_n must be 128 or 256");
  CUtensorMap ta = a_mn ? make_map(a.data_ptr(), M, K, batch, lda, bsa, 64) : make_map(a.data_ptr(), K, M, batch, lda, bsa, BM);
  CUtensorMap tb = b_mn ? make_map(b.data_ptr(), N, K, batch, ldb, bsb, 64) : make_map(b.data_ptr(), K, N, batch, ldb, bsb, BN);
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)batch;
  p.m_tiles = (int)((M + BM - 1) / BM);
  p.n_tiles = (int)((N + BN - 1) / BN);
  p.k_blocks = (int)((K + BK - 1) / BK);
  int splits = (int)std::max<int64_t>(1, k_splits);
  if (k_splits <= 0) {  // auto: fill ~2 waves when the tile count is small, keep >= 8 k-blocks per split
    const int tiles = p.m_tiles * p.n_tiles * p.batch;
    splits = std::max(1, std::min(p.k_blocks / 8, (2 * num_sms() + tiles - 1) / tiles));
    if (epi != EPI_ATOMIC_F32) splits = 1;
  }
  TORCH_CHECK(splits == 1 || epi == EPI_ATOMIC_F32, "k_splits > 1 needs the accumulating epilogue");
  p.kb_per_split = (p.k_blocks + splits - 1) / splits;
  p.k_splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  p.C = c.data_ptr();
  p.ldc = ldc;
  p.bsc = bsc;
  if (aux.has_value() && aux->defined()) {
    p.aux = aux->data_ptr();
    p.ld_aux = ld_aux;
    p.bs_aux = bs_aux;
  }
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.status = status_ptr(a.device().index());
  const int total = p.m_tiles * p.n_tiles * p.batch * p.k_splits;
  const int grid = std::min(total, num_sms());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (BN == 256)
    dispatch_major<256>(a_mn, b_mn, (int)epi, ta, tb, p, grid, st);
  else
    dispatch_major<128>(a_mn, b_mn, (int)epi, ta, tb, p, grid, st);
}

}  // namespace br
