// Persistent warp-specialised tcgen05 GEMM for sm_100a: C[b] = epilogue(A[b] . B[b]^T).
//
//   A: logical [M, K], either K-major (stored [M, K]) or MN-major (stored [K, M]).
//   B: logical [N, K], either K-major (stored [N, K]) or MN-major (stored [K, N]).
//   bf16 operands, fp32 accumulation in TMEM, 128 x BN x 64 tiles (BN = 128 or 256).
//
// Roles (192 threads, or 320 with eight epilogue warps; one CTA per SM, grid = min(work units, SMs)):
//   warp 0  one elected lane issues TMA loads (128-byte swizzle, no multicast) into a
//           STAGES-deep ring of shared-memory stages guarded by full/empty mbarriers;
//   warp 1  allocates TMEM (two BN-column fp32 accumulators) and one elected lane issues
//           tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit;
//   warps 2-5 (2-9)  epilogue. Warp w owns TMEM lanes / tile rows 32*(w%4) .. +31 (with eight warps
//           the two warps of a lane quadrant take one half of the tile's chunks each). Per chunk of 128 bytes
//           of output row (64 bf16 or 32 fp32 columns) it reads the accumulator with tcgen05.ld,
//           applies the fused epilogue, writes the 32 x 128 B chunk into a double-buffered, 128-byte
//           swizzled staging tile in shared memory and issues one TMA store (or TMA reduce-add for
//           split-K) for it. Auxiliary inputs (residual, saved activation) arrive by TMA load into
//           the same staging tile. TMA bounds-checks the M/N edges. The accumulator is released to
//           the MMA warp after the last tcgen05.ld of a tile, so the next tile's main loop overlaps
//           the remaining stores.
// Work units are (k-split, n-tile, m-tile, batch) with n fastest so CTAs running at the same time
// share A rows through L2. With k_splits > 1 each unit reduce-adds its fp32 partial into C (weight
// gradients, whose reduction dimension is the token count).
//
// All mbarrier waits are bounded (2 s); on timeout the kernel records a status code, drains its
// in-flight TMA loads, MMAs and stores, frees TMEM and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "status.h"
#include "tma_host.h"

namespace br {

enum GemmEpi : int {
  EPI_BF16 = 0,        // C(bf16) = alpha*acc + beta*aux(bf16, optional)
  EPI_F32 = 1,         // C(f32)  = alpha*acc + beta*aux(f32, optional; may alias C)
  EPI_RELU2 = 2,       // C(bf16) = relu(alpha*acc)^2
  EPI_RELU2_BWD = 3,   // C(bf16) = alpha*acc * 2*sqrt(aux(bf16))   (d/du of relu(u)^2 given h = relu(u)^2)
  EPI_ATOMIC_F32 = 4,  // C(f32) += alpha*acc                       (TMA reduce-add)
  EPI_SOFTCAP = 5,     // C(bf16) = beta*tanh(alpha*acc)             (alpha = 1/cap, beta = cap)
  EPI_QKV_ROPE = 6,    // fused QKV projection output (see QkvRope), BN = 256
  EPI_SOFTCAP_CE = 7,  // lm_head + softcap + cross-entropy statistics (see CeHead), BN = 256
};

// The QKV projection's epilogue: the output columns are [q heads | k heads | v heads] of 128 columns
// each, and a 256-column tile holds exactly two heads (H and KV even). Per row of a q/k head: half-split
// RoPE (y1 = x1 c + x2 s, y2 = -x1 s + x2 c with c, s = cos/sin tables [T, 64] at the row's position)
// then RMSNorm over the 128 head dims (QK-norm after RoPE, gpt.ts:159-177, :239-244), saving the rstd.
// Per row of a v head on value-embedding layers: v += ve[idx] * 2 sigmoid(cur[:, :32] . Wg[:, h])
// (gpt.ts:225-236), saving the gate.
struct QkvRope {
  const float* cosT;
  const float* sinT;
  float* rq;             // [M, H]
  float* rk;             // [M, KV]
  const int* idx;        // token ids [M]             (value-embedding layers only, else null)
  const float* ve;       // [V, KV*128] fp32 table
  const float* cur;      // [M, ld_cur] ladder output (the gate reads its first 32 columns)
  const float* wg;       // [32, KV]
  float* gate;           // [M, KV]
  int T, H, KV, ld_cur;
  int V;                 // rows of the value-embedding table (token ids are checked against it)
};

// The lm_head epilogue fused with the softcapped cross-entropy (gpt.ts:296-313). With z = cap*tanh(acc/cap)
// every logit lies in [-cap, cap], so e = exp(z - cap) lies in [exp(-2 cap), 1] and needs no running
// maximum. Per element the epilogue writes (when `store`) the bf16 tile of
//   G = e * (1 - (z/cap)^2)          (softmax numerator times the softcap derivative; 0 at the target),
// which the backward GEMMs consume in place of dlogits, and per row and 256-column tile it writes the
// partial sum of e into partial[n_tile][row] and, in the tile holding the row's target, z there.
// `ce_finalize` (loss.cu) turns these into the loss, per-token nats, a per-row scale for G and the
// target column's exact fp32 gradient; the logits themselves are never written.
struct CeHead {
  const int* targets;  // [M] (rows whose target is outside [0, N) are masked)
  float* partial;      // [2 n_tiles][M]: per 256-column tile, the sums over its two halves
  float* zt;           // [M]
  int store;           // 0: statistics only (evaluation)
};

struct GemmParams {
  int M, N, K, batch;
  int k_splits, kb_per_split;
  int m_tiles, n_tiles, k_blocks;
  int has_aux;
  float alpha, beta;
  int* status;
  QkvRope rope;
  CeHead ce;
};

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int CHUNK_BYTES = 32 * 128;  // one epilogue warp's 32 rows x 128 bytes
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

// AUX: the epilogue reads an auxiliary input. Its loads then run through a 5-buffer ring per
// epilogue warp, issued up to three chunks (across tile boundaries) ahead of the chunk being
// processed, so the DRAM latency of the aux tile overlaps the epilogue math. A buffer is reloaded only
// once the store of the chunk two back has read it: the latest chunk's store stays in flight. The
// main loop gives up one stage to make room.
// CG = 2: a CTA pair runs one 256-row tile (cta_group::2); each CTA loads its 128 rows of A and half of
// B's BN columns, so a stage is 32 KB instead of 48 and the pair reads a third less operand data per
// output than two single CTAs.
// EW: epilogue warps. A CTA pair with an aux input, or computing the cross-entropy statistics, runs
// eight, two per TMEM lane quadrant, each taking half of a tile's chunks: with one warp per SM
// sub-partition those epilogues were issue-bound (every TMEM load, aux wait, MUFU op and store of the
// chain exposed), and the pair's smaller stages leave room for the second set of staging buffers.
constexpr int epi_warps(int epi, bool aux, int cg) { return cg == 2 && (aux || epi == EPI_SOFTCAP_CE) ? 8 : 4; }

template <int BN, bool AUX, int CG = 1, int EW_ = 4>
struct GemmCfg {
  static constexpr int EW = EW_;
  static constexpr int THREADS = 64 + 32 * EW;
  static constexpr int STAGES =
      CG == 2 ? (AUX ? 4 : (EW == 8 ? 5 : 6)) : (AUX ? (BN == 256 ? 3 : 4) : (BN == 256 ? 4 : 6));
  // staging buffers per epilogue warp; with an aux input the ring holds the aux loads NBUF - 2 chunks
  // ahead plus the latest chunk's store, so a prefetch never waits for the store it follows
  static constexpr int NBUF = AUX ? (EW == 8 ? 3 : 5) : 2;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / CG) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_BYTES = EW * NBUF * CHUNK_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES + 1024 /*align*/;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert((2 * STAGES + 5 + EW * NBUF) * 8 + 8 <= BAR_BYTES, "barrier region");
};

constexpr bool epi_f32(int e) { return e == EPI_F32 || e == EPI_ATOMIC_F32; }
constexpr bool epi_reads_aux(int e) { return e == EPI_BF16 || e == EPI_F32 || e == EPI_RELU2_BWD; }

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

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* m, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Waits until at most n bulk store groups still read shared memory (n clamped to [0, 2]; waiting for
// fewer pending groups than allowed is always safe).
__device__ __forceinline__ void bulk_wait_read_n(int n) {
  if (n <= 0)
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  else if (n == 1)
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
  else
    asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled staging tile.
__device__ __forceinline__ int swz_off(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Epilogue math on 8 values (one 16-byte bf16 chunk or two fp32 chunks), aux values already unpacked.
template <int EPI>
__device__ __forceinline__ float epi_op(float acc, float aux, const GemmParams& p) {
  if constexpr (EPI == EPI_RELU2_BWD) {
    // aux = h = relu(u)^2 >= 0, so 2 relu(u) = 2 sqrt(h); (2 alpha) is loop-invariant
    return (acc * (2.f * p.alpha)) * sqrt_approx(aux);
  }
  float v = acc * p.alpha;
  if constexpr (EPI == EPI_BF16 || EPI == EPI_F32) {
    v += p.beta * aux;
  } else if constexpr (EPI == EPI_RELU2) {
    v = fmaxf(v, 0.f);
    v = v * v;
  } else if constexpr (EPI == EPI_SOFTCAP) {
    v = p.beta * tanh_approx(v);
  }
  return v;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool AUX, int CG>
__global__ void __launch_bounds__(GemmCfg<BN, AUX, CG, epi_warps(EPI, AUX, CG)>::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX, GemmParams p) {
  static_assert(!AUX || epi_reads_aux(EPI), "aux ring for an epilogue without aux");
  static_assert(CG == 1 || (CG == 2 && BN == 256), "CTA pairs run 256-column tiles");
  using Cfg = GemmCfg<BN, AUX, CG, epi_warps(EPI, AUX, CG)>;
  constexpr int NBUF = Cfg::NBUF;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int EW = Cfg::EW;
  static_assert(EW == 4 || EPI != EPI_QKV_ROPE, "the QKV epilogue uses 4 warps");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sE = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sE + Cfg::EPI_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint64_t* drain_bar = bars + 2 * STAGES + 4;
  uint64_t* aux_bar = bars + 2 * STAGES + 5;  // [EW][NBUF]: per epilogue warp, one per staging buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5 + EW * NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int total = p.m_tiles * p.n_tiles * p.batch * p.k_splits;
  // CTA pairs: the pair shares one work unit (m counts 256-row tiles); rank 0 leads (issues the MMAs)
  const uint32_t crank = CG == 2 ? cluster_rank() : 0u;
  const bool lead = crank == 0;
  const int unit0 = CG == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustride = CG == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  auto row_base = [&](int m) { return (CG == 2 ? 2 * m + (int)crank : m) * BM; };

  // an early return is for single CTAs only: a pair must reach its cluster barriers together
  if constexpr (CG == 1) {
    if (device_failed(p.status)) return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * EW * CG);  // every epilogue thread of the pair releases the leader's
    }
    mbar_init(drain_bar, 1);
    for (int w = 0; w < EW * NBUF; ++w) mbar_init(&aux_bar[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (CG == 2)
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    else
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA arrive or load
  else
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
      // a pair's loads of one stage all count on the leader's full barrier, which expects both halves
      auto load = [&](const CUtensorMap* m, void* dst, int c0, int c1, int c2) {
        if constexpr (CG == 2)
          tma_load_3d_pair(m, &full_bar[stage], dst, c0, c1, c2);
        else
          tma_load_3d(m, &full_bar[stage], dst, c0, c1, c2);
      };
      constexpr int BNC = BN / CG;  // B columns this CTA loads
      for (int u = unit0; u < total && ok; u += ustride) {
        int m, n, b, kb0, kb1;
        decode_unit(p, u, m, n, b, kb0, kb1);
        const int arow = row_base(m);
        const int bcol = n * BN + (int)crank * BNC;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, kWaitBudgetNs, abort_flag, p.status)) {
            fail(kErrTimeoutProducer);
            ok = false;
            break;
          }
          if (CG == 1 || lead) mbar_arrive_expect_tx(&full_bar[stage], CG * Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          if constexpr (!A_MN) {
            load(&tmA, a_dst, kb * BK, arow, b);
          } else {
            load(&tmA, a_dst, arow, kb * BK, b);
            load(&tmA, a_dst + 8192, arow + 64, kb * BK, b);
          }
          if constexpr (!B_MN) {
            load(&tmB, b_dst, kb * BK, bcol, b);
          } else {
#pragma unroll
            for (int j = 0; j < BNC / 64; ++j) load(&tmB, b_dst + j * 8192, bcol + j * 64, kb * BK, b);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // on an early exit, let the issued loads land (a pair's follower cannot see its loads complete: they
      // count on the leader's barrier, whose drain covers them before the final cluster barrier)
      if ((!ok || *abort_flag) && (CG == 1 || lead)) {
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
    if (elect_one() && (CG == 1 || lead)) {  // a pair's follower issues no MMA
      constexpr uint32_t idesc = umma_idesc_bf16(CG * BM, BN, A_MN, B_MN);
      auto mma = [&](uint32_t d, uint64_t ad, uint64_t bd, uint32_t acc) {
        if constexpr (CG == 2)
          umma_bf16_ss_pair(d, ad, bd, idesc, acc);
        else
          umma_bf16_ss(d, ad, bd, idesc, acc);
      };
      auto commit = [&](uint64_t* bar) {
        if constexpr (CG == 2)
          umma_commit_pair(bar);  // the same barrier in both CTAs
        else
          umma_commit(bar);
      };
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = unit0; u < total && ok; u += ustride, ++local) {
        int m, n, b, kb0, kb1;
        decode_unit(p, u, m, n, b, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, kWaitBudgetNs, abort_flag, p.status)) {
          fail(kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kWaitBudgetNs, abort_flag, p.status)) {
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
            mma(d_tmem, ad, bd, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) commit(&tfull_bar[acc]);
      }
      commit(drain_bar);
      mbar_wait(drain_bar, 0, 100000000ull, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps 2..EW+1
    // a warp reads TMEM lanes 32 (warp % 4) .. + 31; with eight warps the two of a quadrant split the
    // tile's chunks into halves (eh = 0, 1)
    const int ew = warp - 2;
    const int wq = warp & 3;
    const int eh = ew >> 2;
    const int lane = lane_id();
    const bool leader = lane == 0;
    uint8_t* ebuf = sE + ew * NBUF * CHUNK_BYTES;
    uint64_t* xbar = &aux_bar[ew * NBUF];
    constexpr int COLS = epi_f32(EPI) ? 32 : 64;  // columns per 128-byte chunk
    constexpr int CPT = BN / COLS;                 // chunks per tile
    constexpr int CPW = CPT / (EW / 4);            // chunks per tile of one warp
    static_assert(CPW * (EW / 4) == CPT, "chunks split evenly between a quadrant's warps");
    const int c_lo = eh * CPW;                     // this warp's first chunk of every tile
    int nchunk = 0;                                // chunks this warp has processed (ring position)
    // aux prefetch cursor (AUX only): next chunk to load, its work unit and chunk within the tile
    int pchunk = 0, pu = unit0, pc = c_lo;
    auto prefetch = [&](int upto) {
      while (pchunk < upto && pu < total) {
        if (pchunk >= NBUF) {
          // buffer pchunk % NBUF last staged chunk pchunk - NBUF: its store must have read it; the
          // stores of the chunks after it may still be pending (one bulk group per chunk)
          const int newer = nchunk - 1 - (pchunk - NBUF);
          if (leader) bulk_wait_read_n(newer);
        }
        if (leader) {
          int m, n, b, kb0, kb1;
          decode_unit(p, pu, m, n, b, kb0, kb1);
          const int slot = pchunk % NBUF;
          mbar_arrive_expect_tx(&xbar[slot], CHUNK_BYTES);
          tma_load_3d(&tmX, &xbar[slot], ebuf + slot * CHUNK_BYTES, n * BN + pc * COLS, row_base(m) + wq * 32, b);
        }
        ++pchunk;
        if (++pc == c_lo + CPW) {
          pc = c_lo;
          pu += ustride;
        }
      }
    };
    int local = 0;
    if (leader) {
      tma_prefetch_desc(&tmC);
      if constexpr (AUX) tma_prefetch_desc(&tmX);
    }
    bool ok = true;
    // hands the accumulator back to the MMA warp (in a pair: on the leader's barrier)
    auto release_acc = [&](int acc) {
      if constexpr (CG == 2) {
        if (lead)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_cluster(cluster_map(&tempty_bar[acc], 0));
      } else {
        mbar_arrive(&tempty_bar[acc]);
      }
    };
    for (int u = unit0; u < total && ok; u += ustride, ++local) {
      int m, n, b, kb0, kb1;
      decode_unit(p, u, m, n, b, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if constexpr (AUX) prefetch(nchunk + NBUF - 1);  // aux of the coming chunks loads during the MMA
      if (!mbar_wait_warp(&tfull_bar[acc], acc_phase, kWaitBudgetNs, abort_flag, p.status)) {
        fail(kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      const int row0 = row_base(m) + wq * 32;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + acc * BN;
      if constexpr (EPI == EPI_QKV_ROPE) {
        // two heads per tile; thread = row. Each head: 128 accumulator columns -> RoPE + QK-norm
        // (q, k heads) or the value-embedding add (v heads) -> two 64-column bf16 chunks.
        const QkvRope& rp = p.rope;
        const int mrow = row0 + lane;
        const bool valid = mrow < p.M;
        const int64_t msafe = valid ? mrow : 0;
        const int nqk = rp.H + rp.KV;
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          const int head = n * 2 + hh;
          uint32_t v[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(taddr + hh * 128 + c * 32, v[c]);
          tmem_ld_wait();
          if (hh == 1) {  // accumulator fully read: hand it back to the MMA warp
            tc_fence_before();
            release_acc(acc);
          }
          float x[128];
#pragma unroll
          for (int i = 0; i < 128; ++i) x[i] = __uint_as_float(v[i >> 5][i & 31]);
          if (head < nqk) {
            const float4* cr = reinterpret_cast<const float4*>(rp.cosT + (int64_t)(mrow % rp.T) * 64);
            const float4* sr = reinterpret_cast<const float4*>(rp.sinT + (int64_t)(mrow % rp.T) * 64);
            float ss = 0.f;
#pragma unroll
            for (int j4 = 0; j4 < 16; ++j4) {
              const float4 c4 = __ldg(cr + j4), s4 = __ldg(sr + j4);
              const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int j = 4 * j4 + k;
                const float x1 = x[j], x2 = x[64 + j];
                const float y1 = x1 * cc[k] + x2 * sn[k], y2 = x2 * cc[k] - x1 * sn[k];
                x[j] = y1;
                x[64 + j] = y2;
                ss = fmaf(y1, y1, fmaf(y2, y2, ss));
              }
            }
            const float r = rsqrtf(ss * (1.f / 128.f) + 1e-5f);
#pragma unroll
            for (int i = 0; i < 128; ++i) x[i] *= r;
            if (valid) {
              if (head < rp.H) rp.rq[(int64_t)mrow * rp.H + head] = r;
              else rp.rk[(int64_t)mrow * rp.KV + (head - rp.H)] = r;
            }
          } else if (rp.ve != nullptr && index_ok(__ldg(rp.idx + msafe), rp.V, valid ? p.status : nullptr)) {
            const int kvh = head - nqk;
            const float4* cz = reinterpret_cast<const float4*>(rp.cur + msafe * rp.ld_cur);
            float z = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 cv = __ldg(cz + c4);
              z = fmaf(cv.x, __ldg(rp.wg + (4 * c4 + 0) * rp.KV + kvh), z);
              z = fmaf(cv.y, __ldg(rp.wg + (4 * c4 + 1) * rp.KV + kvh), z);
              z = fmaf(cv.z, __ldg(rp.wg + (4 * c4 + 2) * rp.KV + kvh), z);
              z = fmaf(cv.w, __ldg(rp.wg + (4 * c4 + 3) * rp.KV + kvh), z);
            }
            const float g = 2.f / (1.f + __expf(-z));
            const float4* e =
                reinterpret_cast<const float4*>(rp.ve + (int64_t)__ldg(rp.idx + msafe) * (rp.KV * 128) + kvh * 128);
#pragma unroll
            for (int d4 = 0; d4 < 32; ++d4) {
              const float4 ev = __ldg(e + d4);
              x[4 * d4 + 0] = fmaf(ev.x, g, x[4 * d4 + 0]);
              x[4 * d4 + 1] = fmaf(ev.y, g, x[4 * d4 + 1]);
              x[4 * d4 + 2] = fmaf(ev.z, g, x[4 * d4 + 2]);
              x[4 * d4 + 3] = fmaf(ev.w, g, x[4 * d4 + 3]);
            }
            if (valid) rp.gate[(int64_t)mrow * rp.KV + kvh] = g;
          }
#pragma unroll
          for (int hc = 0; hc < 2; ++hc, ++nchunk) {
            uint8_t* buf = ebuf + (nchunk & 1) * CHUNK_BYTES;
            if (leader) bulk_wait_read1();  // the store that last used this buffer has read it
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float* xs = x + 64 * hc + 8 * q;
              *reinterpret_cast<uint4*>(buf + swz_off(lane, q)) =
                  make_uint4(pack_bf16(xs[0], xs[1]), pack_bf16(xs[2], xs[3]), pack_bf16(xs[4], xs[5]),
                             pack_bf16(xs[6], xs[7]));
            }
            fence_async_smem();
            __syncwarp();
            if (leader) {
              tma_store_3d(&tmC, buf, n * BN + hh * 128 + hc * 64, row0, b);
              bulk_commit();
            }
          }
        }
        continue;
      }
      // softcapped cross-entropy statistics of this thread's row over the tile (EPI_SOFTCAP_CE)
      float ce_sum = 0.f, ce_zt = 0.f;
      int ce_t = -1;
      if constexpr (EPI == EPI_SOFTCAP_CE) {
        const int mrow = row0 + lane;
        ce_t = mrow < p.M ? __ldg(p.ce.targets + mrow) : -1;
      }
#pragma unroll 1
      for (int c = c_lo; c < c_lo + CPW; ++c, ++nchunk) {
        const int slot = nchunk % NBUF;
        uint8_t* buf = ebuf + slot * CHUNK_BYTES;
        const int col0 = n * BN + c * COLS;
        uint32_t r[COLS];
        tmem_ld32(taddr + c * COLS, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if constexpr (COLS == 64) tmem_ld32(taddr + c * COLS + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        if constexpr (AUX) {
          prefetch(nchunk + NBUF - 1);  // keeps NBUF - 2 chunks ahead in flight; waits only for older stores
        } else {
          if (leader) bulk_wait_read1();  // the store that last used this buffer has read it
        }
        __syncwarp();
        tmem_ld_wait();
        if constexpr (AUX) {
          if (!mbar_wait_warp(&xbar[slot], (nchunk / NBUF) & 1, kWaitBudgetNs, abort_flag, p.status)) {
            fail(kErrTimeoutEpilogue);
            ok = false;
            break;
          }
        }
        uint8_t* myrow = buf;  // row `lane` of this warp's 32-row chunk
        // EPI_SOFTCAP_CE: a chunk inside [0, N) holding no lane's target column (most of them) skips the
        // per-element bounds and target selects
        bool ce_plain = false;
        if constexpr (EPI == EPI_SOFTCAP_CE)
          ce_plain = col0 + COLS <= p.N && !__any_sync(0xffffffffu, ce_t >= col0 && ce_t < col0 + COLS);
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // eight 16-byte chunks per 128-byte row
          uint4* slotp = reinterpret_cast<uint4*>(myrow + swz_off(lane, q));
          if constexpr (EPI == EPI_SOFTCAP_CE) {
            // z = cap tanh(acc/cap); e = exp(z - cap) = 2^((th - 1) cap log2(e)); G = e (1 - th^2)
            const float k2 = p.beta * 1.4426950408889634f;
            uint32_t os[4];
            if (ce_plain) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float g[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const float th = tanh_approx(__uint_as_float(r[8 * q + 2 * j + h]) * p.alpha);
                  const float e = exp2f(fmaf(th, k2, -k2));
                  ce_sum += e;
                  g[h] = e * fmaf(-th, th, 1.f);
                }
                os[j] = pack_bf16(g[0], g[1]);
              }
              *slotp = make_uint4(os[0], os[1], os[2], os[3]);
              continue;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float g[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int col = col0 + 8 * q + 2 * j + h;
                const float th = tanh_approx(__uint_as_float(r[8 * q + 2 * j + h]) * p.alpha);
                const float e = col < p.N ? exp2f(fmaf(th, k2, -k2)) : 0.f;  // TMA zero-fills past N
                ce_sum += e;
                const bool at_t = col == ce_t;
                ce_zt = at_t ? th * p.beta : ce_zt;
                g[h] = at_t ? 0.f : e * fmaf(-th, th, 1.f);
              }
              os[j] = pack_bf16(g[0], g[1]);
            }
            *slotp = make_uint4(os[0], os[1], os[2], os[3]);
          } else if constexpr (epi_f32(EPI)) {
            float4 x = AUX ? *reinterpret_cast<const float4*>(slotp) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 o;
            o.x = epi_op<EPI == EPI_ATOMIC_F32 ? EPI_BF16 : EPI>(__uint_as_float(r[4 * q + 0]), x.x, p);
            o.y = epi_op<EPI == EPI_ATOMIC_F32 ? EPI_BF16 : EPI>(__uint_as_float(r[4 * q + 1]), x.y, p);
            o.z = epi_op<EPI == EPI_ATOMIC_F32 ? EPI_BF16 : EPI>(__uint_as_float(r[4 * q + 2]), x.z, p);
            o.w = epi_op<EPI == EPI_ATOMIC_F32 ? EPI_BF16 : EPI>(__uint_as_float(r[4 * q + 3]), x.w, p);
            *reinterpret_cast<float4*>(slotp) = o;
          } else {
            uint4 xv = AUX ? *slotp : make_uint4(0, 0, 0, 0);
            const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
            uint32_t os[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = unpack_bf16(xs[j]);
              os[j] = pack_bf16(epi_op<EPI>(__uint_as_float(r[8 * q + 2 * j]), f.x, p),
                                epi_op<EPI>(__uint_as_float(r[8 * q + 2 * j + 1]), f.y, p));
            }
            *slotp = make_uint4(os[0], os[1], os[2], os[3]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (c == c_lo + CPW - 1) {
          // accumulator fully read: hand it back to the MMA warp
          tc_fence_before();
          release_acc(acc);
        }
        if (leader && (EPI != EPI_SOFTCAP_CE || p.ce.store)) {
          if constexpr (EPI == EPI_ATOMIC_F32)
            tma_reduce_add_3d(&tmC, buf, col0, row0, b);
          else
            tma_store_3d(&tmC, buf, col0, row0, b);
          bulk_commit();
        }
      }
      if constexpr (EPI == EPI_SOFTCAP_CE) {
        // two partial rows per 256-column tile, one per half of its chunks (with four epilogue warps
        // the second holds 0), so the layout does not depend on the launch form
        const int mrow = row0 + lane;
        if (ok && mrow < p.M) {
          const int cbeg = n * BN + c_lo * COLS;
          p.ce.partial[(int64_t)(2 * n + eh) * p.M + mrow] = ce_sum;
          if constexpr (EW == 4) p.ce.partial[(int64_t)(2 * n + 1) * p.M + mrow] = 0.f;
          if (ce_t >= cbeg && ce_t < cbeg + CPW * COLS) p.ce.zt[mrow] = ce_zt;
        }
      }
    }
    if constexpr (AUX) {
      // on an early exit, let every aux load already issued land before the CTA leaves
      for (int q = nchunk; q < pchunk; ++q) mbar_wait(&xbar[q % NBUF], (q / NBUF) & 1, 100000000ull, nullptr);
    }
    if (leader) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync_all();  // the leader's MMAs and both CTAs' epilogues are done with TMEM and shared memory
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------------- host
namespace {

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

struct Maps {
  CUtensorMap a, b, c, x;
};

// Which 256-column GEMMs with more than one 128-row tile run as CTA pairs (gemm_set_pair, for A/B
// measurements): 0 none; 1 (the default) and 2 all of them. Measured at M = 2^18 against single CTAs:
// ReLU^2 backward (aux, K = 512) 0.612 -> 0.579 ms, MLP projection with residual (aux, K = 2048)
// 0.519 -> 0.493, residual projection (aux, K = 512) 0.245 -> 0.241.
int g_pair = 1;

int pair_mode(int BN, int64_t M) { return BN == 256 && M > BM && g_pair != 0 ? 2 : 1; }

// Persistent grid: one CTA (or one CTA pair) per SM (pair), no more than there are work units.
int persistent_grid(int64_t units, int cg) {
  const int slots = num_sms() / cg;
  return cg * (int)std::min<int64_t>(units, slots);
}

template <int BN, bool AMN, bool BMN, int EPI, bool AUX, int CG>
void launch_cg(const Maps& mp, const GemmParams& p, int grid, cudaStream_t st) {
  auto k = gemm_kernel<BN, AMN, BMN, EPI, AUX, CG>;
  using Cfg = GemmCfg<BN, AUX, CG, epi_warps(EPI, AUX, CG)>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    attr = true;
  }
  if constexpr (CG == 1) {
    k<<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(mp.a, mp.b, mp.c, mp.x, p);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    // a persistent pair grid no larger than the pairs that can be resident at once (SM pairs of a GPC)
    static int max_pairs = 0;
    if (!max_pairs) {
      cfg.gridDim = dim3((unsigned)grid);
      C10_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&max_pairs, k, &cfg));
      if (max_pairs < 1) max_pairs = 1;
    }
    cfg.gridDim = dim3((unsigned)std::min(grid, 2 * max_pairs));
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, mp.a, mp.b, mp.c, mp.x, p));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, bool AMN, bool BMN, int EPI, bool AUX>
void launch_t(const Maps& mp, const GemmParams& p, int grid, cudaStream_t st, int cg) {
  if constexpr (BN == 256) {
    if (cg == 2) return launch_cg<BN, AMN, BMN, EPI, AUX, 2>(mp, p, grid, st);
  }
  TORCH_CHECK(cg == 1, "gemm: CTA pairs need 256-column tiles");
  launch_cg<BN, AMN, BMN, EPI, AUX, 1>(mp, p, grid, st);
}

template <int BN, bool AMN, bool BMN>
void dispatch_epi(int epi, const Maps& mp, const GemmParams& p, int grid, cudaStream_t st, int cg) {
  const bool aux = p.has_aux != 0;
  switch (epi) {
    case EPI_BF16:
      return aux ? launch_t<BN, AMN, BMN, EPI_BF16, true>(mp, p, grid, st, cg)
                 : launch_t<BN, AMN, BMN, EPI_BF16, false>(mp, p, grid, st, cg);
    case EPI_F32:
      return aux ? launch_t<BN, AMN, BMN, EPI_F32, true>(mp, p, grid, st, cg)
                 : launch_t<BN, AMN, BMN, EPI_F32, false>(mp, p, grid, st, cg);
    case EPI_ATOMIC_F32: return launch_t<BN, AMN, BMN, EPI_ATOMIC_F32, false>(mp, p, grid, st, cg);
    default: break;
  }
  if constexpr (BN == 256) {
    switch (epi) {
      case EPI_RELU2: return launch_t<BN, AMN, BMN, EPI_RELU2, false>(mp, p, grid, st, cg);
      case EPI_RELU2_BWD: return launch_t<BN, AMN, BMN, EPI_RELU2_BWD, true>(mp, p, grid, st, cg);
      case EPI_SOFTCAP: return launch_t<BN, AMN, BMN, EPI_SOFTCAP, false>(mp, p, grid, st, cg);
      default: break;
    }
  }
  TORCH_CHECK(false, "unsupported gemm epilogue ", epi, " for BN=", BN);
}

template <int BN>
void dispatch_major(bool amn, bool bmn, int epi, const Maps& mp, const GemmParams& p, int grid, cudaStream_t st,
                    int cg) {
  if (!amn && !bmn) return dispatch_epi<BN, false, false>(epi, mp, p, grid, st, cg);
  if (!amn && bmn) return dispatch_epi<BN, false, true>(epi, mp, p, grid, st, cg);
  if (amn && !bmn) return dispatch_epi<BN, true, false>(epi, mp, p, grid, st, cg);
  return dispatch_epi<BN, true, true>(epi, mp, p, grid, st, cg);
}

CUtensorMap bf16_map(const void* base, int64_t inner, int64_t outer, int64_t batch, int64_t ld, int64_t bs, int box_outer) {
  return tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, inner, outer, batch, ld, bs, 64, box_outer);
}

// map for the epilogue's 32-row x 128-byte chunks of an [batch][M][N] tensor
CUtensorMap out_map(const torch::Tensor& t, int64_t M, int64_t N, int64_t batch, int64_t ld, int64_t bs) {
  if (t.scalar_type() == at::kFloat)
    return tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, t.data_ptr(), N, M, batch, ld, bs, 32, 32);
  return tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), N, M, batch, ld, bs, 64, 32);
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
  c10::cuda::CUDAGuard guard(a.device());
  const int BN = block_n > 0 ? (int)block_n : (N <= 128 ? 128 : 256);
  TORCH_CHECK(BN == 128 || BN == 256, "block_n must be 128 or 256");
  Maps mp;
  mp.a = a_mn ? bf16_map(a.data_ptr(), M, K, batch, lda, bsa, 64) : bf16_map(a.data_ptr(), K, M, batch, lda, bsa, BM);
  // a CTA pair loads half of B's tile columns each
  const int cg = pair_mode(BN, M);
  mp.b = b_mn ? bf16_map(b.data_ptr(), N, K, batch, ldb, bsb, 64)
              : bf16_map(b.data_ptr(), K, N, batch, ldb, bsb, BN / cg);
  mp.c = out_map(c, M, N, batch, ldc, bsc);
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)batch;
  p.m_tiles = (int)((M + BM * cg - 1) / (BM * cg));
  p.n_tiles = (int)((N + BN - 1) / BN);
  p.k_blocks = (int)((K + BK - 1) / BK);
  int splits = (int)std::max<int64_t>(1, k_splits);
  if (k_splits <= 0) {
    // auto split-K: among split counts that keep >= 16 k-blocks per split, pick the one whose work
    // units fill the persistent grid's waves best (least idle fraction in the last wave), preferring
    // fewer splits (less reduce-add traffic) on ties
    const int tiles = p.m_tiles * p.n_tiles * p.batch;
    const int sms = num_sms() / cg;  // persistent slots: SMs, or SM pairs
    splits = 1;
    double best = 1e9;
    const int max_s = std::max(1, std::min(64, p.k_blocks / 16));
    for (int sp = 1; sp <= max_s; ++sp) {
      const int64_t units = (int64_t)tiles * sp;
      const int64_t waves = (units + sms - 1) / sms;
      const double waste = (double)(waves * sms - units) / (double)(waves * sms);
      const double cost = waste + (units < sms ? 1.0 : 0.0) + 0.002 * sp;
      if (cost < best - 1e-9) {
        best = cost;
        splits = sp;
      }
    }
    if (epi != EPI_ATOMIC_F32) splits = 1;
  }
  TORCH_CHECK(splits == 1 || epi == EPI_ATOMIC_F32, "k_splits > 1 needs the accumulating epilogue");
  p.kb_per_split = (p.k_blocks + splits - 1) / splits;
  p.k_splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  if (aux.has_value() && aux->defined()) {
    TORCH_CHECK(aux->scalar_type() == c.scalar_type(), "gemm: aux dtype must match the output");
    TORCH_CHECK(epi == EPI_BF16 || epi == EPI_F32 || epi == EPI_RELU2_BWD, "gemm: this epilogue takes no aux");
    mp.x = out_map(*aux, M, N, batch, ld_aux, bs_aux);
    p.has_aux = 1;
  } else {
    TORCH_CHECK(epi != EPI_RELU2_BWD, "gemm: the ReLU^2 backward epilogue needs aux");
    mp.x = mp.c;
    p.has_aux = 0;
  }
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.status = status_ptr(a.device().index());
  const int total = p.m_tiles * p.n_tiles * p.batch * p.k_splits;
  const int grid = persistent_grid(total, cg);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (BN == 256)
    dispatch_major<256>(a_mn, b_mn, (int)epi, mp, p, grid, st, cg);
  else
    dispatch_major<128>(a_mn, b_mn, (int)epi, mp, p, grid, st, cg);
}

// The lm_head GEMM fused with the softcapped cross-entropy statistics (EPI_SOFTCAP_CE, see CeHead):
// x [M, K] bf16 rows, w [N, K] bf16 rows (the [vocab, dim] table), g [M, N] bf16 (written when store),
// targets int32 [M], partial fp32 [2 ceil(N/256), M], zt fp32 [M].
void gemm_softcap_ce(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& g, const torch::Tensor& targets,
                     torch::Tensor& partial, torch::Tensor& zt, double cap, bool store) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && g.scalar_type() == at::kBFloat16,
              "gemm_softcap_ce: bf16 x, w, g");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && g.stride(1) == 1, "gemm_softcap_ce: contiguous rows");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && g.size(0) == M && g.size(1) == N, "gemm_softcap_ce: shapes");
  TORCH_CHECK(targets.scalar_type() == at::kInt && targets.is_contiguous() && targets.numel() == M,
              "gemm_softcap_ce: int32 targets [M]");
  const int64_t n_tiles = (N + 255) / 256;
  TORCH_CHECK(partial.scalar_type() == at::kFloat && partial.is_contiguous() && partial.numel() >= 2 * n_tiles * M,
              "gemm_softcap_ce: partial fp32 [2 ceil(N/256), M]");
  TORCH_CHECK(zt.scalar_type() == at::kFloat && zt.numel() >= M, "gemm_softcap_ce: zt fp32 [M]");
  TORCH_CHECK(cap > 0, "gemm_softcap_ce: cap > 0");
  c10::cuda::CUDAGuard guard(x.device());
  Maps mp;
  mp.a = bf16_map(x.data_ptr(), K, M, 1, x.stride(0), 0, BM);
  const int cg = pair_mode(256, M);
  mp.b = bf16_map(w.data_ptr(), K, N, 1, w.stride(0), 0, 256 / cg);
  mp.c = out_map(g, M, N, 1, g.stride(0), 0);
  mp.x = mp.c;
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = 1;
  p.m_tiles = (int)((M + BM * cg - 1) / (BM * cg));
  p.n_tiles = (int)n_tiles;
  p.k_blocks = (int)((K + BK - 1) / BK);
  p.k_splits = 1;
  p.kb_per_split = p.k_blocks;
  p.has_aux = 0;
  p.alpha = (float)(1.0 / cap);
  p.beta = (float)cap;
  p.status = status_ptr(x.device().index());
  p.ce.targets = targets.data_ptr<int>();
  p.ce.partial = partial.data_ptr<float>();
  p.ce.zt = zt.data_ptr<float>();
  p.ce.store = store ? 1 : 0;
  const int total = p.m_tiles * p.n_tiles;
  launch_t<256, false, false, EPI_SOFTCAP_CE, false>(mp, p, persistent_grid(total, cg),
                                                      at::cuda::getCurrentCUDAStream(), cg);
}

// out[M, (H+2KV)*128] = x[M, K] @ w[K, N] with the QKV epilogue (RoPE + QK-norm on q/k heads, the
// value-embedding add on v heads when `ve` is given). x, w, out: bf16 with contiguous rows.
void gemm_qkv_rope(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, const torch::Tensor& cosT,
                   const torch::Tensor& sinT, torch::Tensor& rq, torch::Tensor& rk, int64_t T, int64_t H, int64_t KV,
                   c10::optional<torch::Tensor> idx, c10::optional<torch::Tensor> ve,
                   c10::optional<torch::Tensor> cur, c10::optional<torch::Tensor> wg,
                   c10::optional<torch::Tensor> gate) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "gemm_qkv_rope: bf16 tensors");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_qkv_rope: contiguous rows");
  TORCH_CHECK(H % 2 == 0 && KV % 2 == 0, "gemm_qkv_rope: even head counts (two heads per 256-column tile)");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(1);
  TORCH_CHECK(w.size(0) == K && N == (H + 2 * KV) * 128 && out.size(0) == M && out.size(1) == N,
              "gemm_qkv_rope: shapes");
  TORCH_CHECK(cosT.scalar_type() == at::kFloat && cosT.is_contiguous() && cosT.size(-1) == 64 &&
                  sinT.is_contiguous() && cosT.numel() >= T * 64, "gemm_qkv_rope: cos/sin tables [T, 64] fp32");
  TORCH_CHECK(rq.numel() >= M * H && rk.numel() >= M * KV, "gemm_qkv_rope: rstd buffers");
  c10::cuda::CUDAGuard guard(x.device());
  Maps mp;
  mp.a = bf16_map(x.data_ptr(), K, M, 1, x.stride(0), 0, BM);
  mp.b = bf16_map(w.data_ptr(), N, K, 1, w.stride(0), 0, 64);
  mp.c = out_map(out, M, N, 1, out.stride(0), 0);
  mp.x = mp.c;
  const int cg = pair_mode(256, M);
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = 1;
  p.m_tiles = (int)((M + BM * cg - 1) / (BM * cg));
  p.n_tiles = (int)(N / 256);
  p.k_blocks = (int)((K + BK - 1) / BK);
  p.k_splits = 1;
  p.kb_per_split = p.k_blocks;
  p.has_aux = 0;
  p.alpha = 1.f;
  p.beta = 0.f;
  p.status = status_ptr(x.device().index());
  QkvRope& r = p.rope;
  r.cosT = cosT.data_ptr<float>();
  r.sinT = sinT.data_ptr<float>();
  r.rq = rq.data_ptr<float>();
  r.rk = rk.data_ptr<float>();
  r.T = (int)T;
  r.H = (int)H;
  r.KV = (int)KV;
  const bool has_ve = ve.has_value() && ve->defined();
  if (has_ve) {
    TORCH_CHECK(idx.has_value() && cur.has_value() && wg.has_value() && gate.has_value(), "gemm_qkv_rope: VE args");
    TORCH_CHECK(idx->scalar_type() == at::kInt && ve->scalar_type() == at::kFloat && cur->scalar_type() == at::kFloat &&
                    wg->scalar_type() == at::kFloat && wg->size(0) == 32 && wg->size(1) == KV,
                "gemm_qkv_rope: VE dtypes/shapes");
    TORCH_CHECK(cur->stride(-1) == 1 && cur->stride(0) % 4 == 0 && ve->size(-1) == KV * 128, "gemm_qkv_rope: VE layout");
    r.idx = idx->data_ptr<int>();
    r.ve = ve->data_ptr<float>();
    r.cur = cur->data_ptr<float>();
    r.ld_cur = (int)cur->stride(0);
    r.wg = wg->data_ptr<float>();
    r.gate = gate->data_ptr<float>();
    r.V = (int)ve->size(0);
  }
  const int total = p.m_tiles * p.n_tiles;
  launch_t<256, false, true, EPI_QKV_ROPE, false>(mp, p, persistent_grid(total, cg), at::cuda::getCurrentCUDAStream(),
                                                  cg);
}

void gemm_set_pair(int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 2, "gemm_set_pair: 0 (none), 1 (the default policy: all) or 2 (all)");
  g_pair = (int)mode;
}
int64_t gemm_pair() { return g_pair; }

}  // namespace br
