// tcgen05/TMEM flash attention for sm_100a (head_dim 128, causal + sliding window).
//
// Forward: persistent, one CTA per SM, 320 threads; a work item is (two 128-query tiles A and B, head,
// batch), taken from a device counter by warp 0 and handed to the other warps (see the kernel):
//   warp 0      TMA: the item's two Q tiles, then K tiles into a 3-stage ring and V tiles into a 2-stage
//               ring (128-byte swizzle, 3-D tensor maps over the fused [B, T, Dq+2Dkv] projection
//               buffer, zero fill past T; no multicast);
//   warp 1      TMEM allocation and the single MMA-issuing lane. Per query tile X:
//                 S_X = Q_X K_t^T  -> TMEM [256X, +128)          (fp32)
//                 P_X              -> TMEM [256X, +64)           (bf16 pairs, written over S_X)
//                 O_X += P_X V_t   -> TMEM [256X + 128, +128)    (A operand read from TMEM)
//               issued in the order S_A S_B | PV_A S_A' PV_B S_B' | ..., so the tensor core works on
//               one tile while the other tile's softmax runs;
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: one query row per thread (TMEM lane =
//               row), masked row max, conditional rescale of O (only when the running max grows by
//               more than 2^8, so P stays below 256), P = exp2(S*scale - m) packed to bf16 and stored
//               back to TMEM; finally O / l and the log-sum-exp.
// S_X(j+1) is issued after PV_X(j), and the tcgen05.mma of one CTA complete in issue order, so when the
// softmax of S_X(j+1) starts, PV_X(j) has finished reading P_X(j) and writing O_X: the softmax may
// overwrite P and rescale O without another barrier.
// Key tiles outside a tile's band [q - w + 1, q] are never loaded. All mbarrier waits are bounded; on
// timeout the CTA records a status code, drains its MMAs, frees TMEM and exits.
//
// Backward: a dQ kernel and a dK/dV kernel (described where they are defined).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <type_traits>

#include "common.cuh"
#include "status.h"
#include "tma_host.h"

namespace br {
namespace {

constexpr int HD = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int TILE_BYTES = 128 * 128 * 2;  // one 128 x 128 bf16 tile (two 64-column swizzle atoms)
constexpr int ATOM_BYTES = 128 * 128;      // 128 rows x 128 bytes
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kBudgetNs = 2000000000ull;

struct FwdParams {
  int B, T, H, KV, Dq, Dkv, window;
  float scale_log2;
  __nv_bfloat16* out;
  int64_t ldo;
  float* lse;
  int* status;
};

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

constexpr int F2_Q = 0;                               // [2] x 32 KB: Q_A, Q_B
constexpr int F2_KST = 3;                             // K ring depth
constexpr int F2_VST = 2;                             // V ring depth
constexpr int F2_K = F2_Q + 2 * TILE_BYTES;           // [3] x 32 KB
constexpr int F2_V = F2_K + F2_KST * TILE_BYTES;      // [2] x 32 KB
constexpr int F2_BAR = F2_V + F2_VST * TILE_BYTES;
constexpr int FWD_SMEM = F2_BAR + 256 + 1024;

struct Band {
  int lo, n;  // first key tile and number of key tiles of a query tile
  __device__ bool uses(int t) const { return t >= lo && t < lo + n; }
};

__device__ __forceinline__ Band band_of(int q0, int T, int w) {
  Band b;
  if (q0 >= T) {
    b.lo = 0;
    b.n = 0;
    return b;
  }
  b.lo = max(0, q0 - w + 1) / BKV;
  const int hi = min(q0 + BQ - 1, T - 1) / BKV;
  b.n = hi - b.lo + 1;
  return b;
}

// Persistent, dynamically scheduled: grid = min(work items, SMs). A CTA's producer takes work items (a
// pair of 128-query tiles, a head, a batch row) from a device counter and hands each to the MMA and
// softmax warps through a two-slot ring in shared memory, so TMEM, barriers and the K/V rings are set up
// once per SM, the next item's Q load and first score MMAs overlap the current item's output epilogue,
// and items of uneven cost (the causal band holds 2 to 18 key tiles per item) balance across SMs as
// they would under the hardware's CTA scheduling. Ring positions and barrier phases run on across
// items. q_empty lets the producer reload the Q tiles once the item's last score MMA has completed;
// o_empty[x] holds query tile x's first PV MMA of an item until the softmax warps have read the previous
// item's O. The last CTA to finish resets the counter for the next launch (launches of this kernel on
// one device must not overlap: they share the counter).
__device__ int g_fwd_sched[2];  // [0] next work item, [1] CTAs finished

struct FwdItem {
  int h, b, kvh, q0, u_lo, nu;
  Band bA, bB;
  bool same_start;
  // Last user of key tile t among the two query tiles, in MMA issue order: when both tiles start at
  // the same key tile, B's MMAs on t come after A's; when B starts one tile later, A's come last.
  __device__ bool last_is_b(int t) const { return same_start ? bB.uses(t) : !bA.uses(t); }
};

__device__ __forceinline__ FwdItem fwd_item(int item, const FwdParams& p) {
  const int n_qp = (p.T + 2 * BQ - 1) / (2 * BQ);
  FwdItem I;
  const int qp = item % n_qp;
  I.h = (item / n_qp) % p.H;
  I.b = item / (n_qp * p.H);
  I.kvh = I.h / (p.H / p.KV);
  I.q0 = qp * 2 * BQ;
  I.bA = band_of(I.q0, p.T, p.window);
  I.bB = band_of(I.q0 + BQ, p.T, p.window);
  // key tiles of the item: bA.lo .. last tile of B (or of A when B is past T)
  I.u_lo = I.bA.lo;
  const int u_hi = I.bB.n > 0 ? I.bB.lo + I.bB.n - 1 : I.bA.lo + I.bA.n - 1;
  I.nu = u_hi - I.u_lo + 1;
  I.same_start = I.bB.n > 0 && I.bB.lo == I.bA.lo;
  return I;
}

// Called once by thread 0 of every CTA on its way out: the last one resets the scheduler.
__device__ __forceinline__ void fwd_sched_exit() {
  __threadfence();
  if (atomicAdd(&g_fwd_sched[1], 1) == (int)gridDim.x - 1) {
    g_fwd_sched[0] = 0;
    g_fwd_sched[1] = 0;
    __threadfence();
  }
}

__global__ void __launch_bounds__(320, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F2_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [3]
  uint64_t* k_empty = bars + 4;  // [3]
  uint64_t* v_full = bars + 7;   // [2]
  uint64_t* v_empty = bars + 9;  // [2]
  uint64_t* s_full = bars + 11;  // [2] per query tile
  uint64_t* p_full = bars + 13;  // [2] per query tile
  uint64_t* o_done = bars + 15;  // [2] per query tile
  uint64_t* drain = bars + 17;
  uint64_t* q_empty = bars + 18;
  uint64_t* o_empty = bars + 19;     // [2] per query tile
  uint64_t* item_full = bars + 21;   // [2] item ring slots
  uint64_t* item_empty = bars + 23;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 25);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* item_ring = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [2]
  static_assert(25 * 8 + 16 <= 256, "forward barrier region");

  const int n_items = ((p.T + 2 * BQ - 1) / (2 * BQ)) * p.H * p.B;
  const int warp = warp_id();
  if (device_failed(p.status)) {
    if (threadIdx.x == 0) fwd_sched_exit();
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < F2_KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < F2_VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 128);
      mbar_init(&o_done[x], 1);
      mbar_init(&o_empty[x], 128);
      mbar_init(&item_full[x], 1);
      mbar_init(&item_empty[x], 9);  // the MMA thread and one lane of each softmax warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) {
    *abort_flag = 1;
    if (p.status) atomicCAS(p.status, 0, code);
  };

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tm);
      int ik = 0, iv = 0;  // K and V tiles loaded so far (ring positions)
      bool ok = true;
      for (int n = 0;; ++n) {
        // take the next work item and publish it (or the end, -1) to the MMA and softmax warps
        const int slot = n & 1;
        if (n >= 2 && !mbar_wait(&item_empty[slot], ((n - 2) >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
          ok = false;
          break;
        }
        int item = atomicAdd(&g_fwd_sched[0], 1);
        if (item >= n_items) item = -1;
        item_ring[slot] = item;
        mbar_arrive(&item_full[slot]);
        if (item < 0) break;
        const FwdItem I = fwd_item(item, p);
        // the previous item's score MMAs have read the Q tiles
        if (n > 0 && !mbar_wait(q_empty, (n - 1) & 1, kBudgetNs, abort_flag, p.status)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
        for (int x = 0; x < 2; ++x) {
          tma_load_3d(&tm, q_full, smem + F2_Q + x * TILE_BYTES, I.h * HD, I.q0 + x * BQ, I.b);
          tma_load_3d(&tm, q_full, smem + F2_Q + x * TILE_BYTES + ATOM_BYTES, I.h * HD + 64, I.q0 + x * BQ, I.b);
        }
        // K runs up to two tiles ahead of V (B's next scores need K[t+1] while A still reads V[t]),
        // so the two rings are filled in one interleaved order: K0, K1, V0, K2, V1, K3, V2, ...
        int lk = 0, lv = 0;
        while (ok && (lk < I.nu || lv < I.nu)) {
          const bool do_k = lk < I.nu && (lk < lv + 2);
          if (do_k) {
            const int st = ik % F2_KST;
            if (!mbar_wait(&k_empty[st], ((ik / F2_KST) & 1) ^ 1, kBudgetNs, abort_flag, p.status)) {
              ok = false;
              break;
            }
            const int k0 = (I.u_lo + lk) * BKV;
            uint8_t* ks = smem + F2_K + st * TILE_BYTES;
            mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
            tma_load_3d(&tm, &k_full[st], ks, p.Dq + I.kvh * HD, k0, I.b);
            tma_load_3d(&tm, &k_full[st], ks + ATOM_BYTES, p.Dq + I.kvh * HD + 64, k0, I.b);
            ++ik;
            ++lk;
          } else {
            const int st = iv % F2_VST;
            if (!mbar_wait(&v_empty[st], ((iv / F2_VST) & 1) ^ 1, kBudgetNs, abort_flag, p.status)) {
              ok = false;
              break;
            }
            const int k0 = (I.u_lo + lv) * BKV;
            uint8_t* vs = smem + F2_V + st * TILE_BYTES;
            mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
            tma_load_3d(&tm, &v_full[st], vs, p.Dq + p.Dkv + I.kvh * HD, k0, I.b);
            tma_load_3d(&tm, &v_full[st], vs + ATOM_BYTES, p.Dq + p.Dkv + I.kvh * HD + 64, k0, I.b);
            ++iv;
            ++lv;
          }
        }
        if (!ok) break;
      }
      if (!ok) fail(kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, 128, false, true);
      int kbase = 0, vbase = 0;            // ring positions of the item's first K and V tiles
      int pc[2] = {0, 0}, oc[2] = {0, 0};  // per query tile: P blocks consumed, items whose O is complete
      bool ok = true;
      for (int n = 0; ok; ++n) {
        const int slot = n & 1;
        if (!mbar_wait(&item_full[slot], (n >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const int item = item_ring[slot];
        mbar_arrive(&item_empty[slot]);
        if (item < 0) break;
        const FwdItem I = fwd_item(item, p);
        const int n_s = I.bA.n + I.bB.n;
        int s_issued = 0;
        ok = mbar_wait(q_full, n & 1, kBudgetNs, abort_flag, p.status);
        // S_X(j) = Q_X K_t^T for key tile t = lo_X + j
        auto issue_s = [&](int x, int j) -> bool {
          const Band& bx = x ? I.bB : I.bA;
          const int t = bx.lo + j, g = kbase + (t - I.u_lo), st = g % F2_KST;
          if (!mbar_wait(&k_full[st], (g / F2_KST) & 1, kBudgetNs, abort_flag, p.status)) return false;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(smem + F2_Q + x * TILE_BYTES);
          const uint32_t k_addr = smem_u32(smem + F2_K + st * TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
            umma_bf16_ss(tmem + x * 256, umma_desc_sw128(q_addr + off, 16, 1024),
                         umma_desc_sw128(k_addr + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[x]);
          if (I.last_is_b(t) == (x == 1)) umma_commit(&k_empty[st]);
          if (++s_issued == n_s) umma_commit(q_empty);  // the item's last score MMA: Q may be reloaded
          return true;
        };
        // O_X += P_X V_t, P from TMEM
        auto issue_pv = [&](int x, int j) -> bool {
          const Band& bx = x ? I.bB : I.bA;
          const int t = bx.lo + j, g = vbase + (t - I.u_lo), st = g % F2_VST;
          // the first PV of an item overwrites O: the softmax warps have read the previous item's
          if (j == 0 && oc[x] > 0 && !mbar_wait(&o_empty[x], (oc[x] - 1) & 1, kBudgetNs, abort_flag, p.status))
            return false;
          if (!mbar_wait(&p_full[x], pc[x] & 1, kBudgetNs, abort_flag, p.status) ||
              !mbar_wait(&v_full[st], (g / F2_VST) & 1, kBudgetNs, abort_flag, p.status))
            return false;
          ++pc[x];
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + F2_V + st * TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_bf16_ts(tmem + x * 256 + 128, tmem + x * 256 + kk * 8,
                         umma_desc_sw128(v_addr + kk * 2048, ATOM_BYTES, 1024), idesc_o,
                         (j > 0 || kk > 0) ? 1u : 0u);
          if (I.last_is_b(t) == (x == 1)) umma_commit(&v_empty[st]);
          if (j == bx.n - 1) {
            umma_commit(&o_done[x]);
            ++oc[x];
          }
          return true;
        };
        if (ok && I.bA.n > 0) ok = issue_s(0, 0);
        if (ok && I.bB.n > 0) ok = issue_s(1, 0);
        for (int j = 0; ok && (j < I.bA.n || j < I.bB.n); ++j) {
          for (int x = 0; x < 2 && ok; ++x) {
            const int nx = x ? I.bB.n : I.bA.n;
            if (j >= nx) continue;
            ok = issue_pv(x, j);
            if (ok && j + 1 < nx) ok = issue_s(x, j + 1);
          }
        }
        kbase += I.nu;
        vbase += I.nu;
      }
      if (!ok) fail(kErrTimeoutMma);
      umma_commit(drain);
      mbar_wait(drain, 0, 100000000ull, nullptr);
    }
  } else {
    // softmax warps: query tile x = (warp - 2) / 4, row r of the tile (TMEM lane group = warp % 4)
    const int x = (warp - 2) >> 2;
    const int wq = warp & 3;
    const int lane = lane_id();
    const int r = wq * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16) + x * 256;
    int sc = 0, oc = 0;  // score blocks consumed and items finished by this query tile
    bool ok = true;
    for (int n = 0; ok; ++n) {
      const int slot = n & 1;
      if (!mbar_wait_warp(&item_full[slot], (n >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
        fail(kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      const int item = item_ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      if (item < 0) break;
      Band bx;
      int qt;
      {
        const FwdItem I = fwd_item(item, p);
        bx = x ? I.bB : I.bA;
        qt = I.q0 + x * BQ;
      }
      const int qi = qt + r;
      const int w = p.window;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < bx.n; ++j, ++sc) {
        if (!mbar_wait_warp(&s_full[x], sc & 1, kBudgetNs, abort_flag, p.status)) {
          fail(kErrTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        const int k0 = (bx.lo + j) * BKV;
        // interior tiles (every key visible to every row of the tile) skip the per-element mask
        const bool interior = (k0 + BKV - 1 <= qt) && (k0 > qt + BQ - 1 - w) && (k0 + BKV <= p.T);
        uint32_t sr[4][32];  // raw S row (masked entries set to -inf)
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(lane_base + c * 32, sr[c]);
        tmem_ld_wait();
        // row max of the raw scores (scale > 0, so it is the max of the scaled ones too); query qi sees
        // key k0 + 32c + i for i in [qi - w + 1 - k0 - 32c, qi + 1 - k0 - 32c) below T - k0 - 32c
        float mx = -INFINITY;
        if (interior) {
#pragma unroll
          for (int i = 0; i < BKV; ++i) mx = fmaxf(mx, __uint_as_float(sr[i >> 5][i & 31]));
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int kc = k0 + 32 * c;
            const uint32_t vis = qi < p.T ? range_mask32(qi - w + 1 - kc, min(qi + 1 - kc, p.T - kc)) : 0u;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float v = ((vis >> i) & 1u) ? __uint_as_float(sr[c][i]) : -INFINITY;
              sr[c][i] = __float_as_uint(v);
              mx = fmaxf(mx, v);
            }
          }
        }
        mx *= p.scale_log2;
        // The rescale decision is per row, but tcgen05.ld/st are warp-collective: the warp rescales
        // together whenever any of its rows needs it, rows that do not use alpha = 1. PV_X(j-1) is
        // complete here (it was issued before S_X(j)).
        float alpha = 1.f;
        bool mine = false;
        if (j == 0) {
          m_ref = mx;
        } else if (mx > m_ref + 8.f) {
          mine = true;
          alpha = m_ref == -INFINITY ? 0.f : exp2f(m_ref - mx);
          l *= alpha;
          m_ref = mx;
        }
        if (__any_sync(0xffffffffu, mine)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld32(lane_base + 128 + c * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st32(lane_base + 128 + c * 32, v);
          }
        }
        // P = exp2(s * scale_log2 - m_ref) -> bf16 pairs into TMEM columns [0, 64) of this tile (masked
        // entries are -inf -> 0); the scale-and-subtract and the row sum run on f32x2 pairs
        const float mref = m_ref == -INFINITY ? 0.f : m_ref;
        const uint64_t sc2 = f32x2(p.scale_log2, p.scale_log2), nm2 = f32x2(-mref, -mref);
        uint64_t l2 = f32x2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const int e = c * 64 + i;
            const float2 t = f32x2_split(fma_f32x2(
                f32x2(__uint_as_float(sr[e >> 5][e & 31]), __uint_as_float(sr[e >> 5][(e + 1) & 31])), sc2, nm2));
            const float p0 = exp2f(t.x), p1 = exp2f(t.y);
            l2 = add_f32x2(l2, f32x2(p0, p1));
            pk[i / 2] = pack_bf16(p0, p1);
          }
          tmem_st32(lane_base + c * 32, pk);
        }
        {
          const float2 ls = f32x2_split(l2);
          l += ls.x + ls.y;
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
      }
      if (bx.n == 0 || !ok) continue;
      if (!mbar_wait_warp(&o_done[x], oc & 1, kBudgetNs, abort_flag, p.status)) {
        fail(kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int hb = item / ((p.T + 2 * BQ - 1) / (2 * BQ));  // b * H + h
      const int h = hb % p.H, b = hb / p.H;
      __nv_bfloat16* orow = p.out + ((int64_t)b * p.T + qi) * p.ldo + h * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_base + 128 + c * 32, v);
        tmem_ld_wait();
        if (qi < p.T) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o;
            o.x = pack_bf16(__uint_as_float(v[8 * q + 0]) * inv, __uint_as_float(v[8 * q + 1]) * inv);
            o.y = pack_bf16(__uint_as_float(v[8 * q + 2]) * inv, __uint_as_float(v[8 * q + 3]) * inv);
            o.z = pack_bf16(__uint_as_float(v[8 * q + 4]) * inv, __uint_as_float(v[8 * q + 5]) * inv);
            o.w = pack_bf16(__uint_as_float(v[8 * q + 6]) * inv, __uint_as_float(v[8 * q + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + q * 8) = o;
          }
        }
      }
      if (qi < p.T) p.lse[(int64_t)hb * p.T + qi] = m_ref + __log2f(l);  // log2 units, [B, H, T]
      // O is read: the next item's first PV MMA of this tile may overwrite it
      tc_fence_before();
      mbar_arrive(&o_empty[x]);
      ++oc;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) fwd_sched_exit();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ------------------------------------------------------------------------------------------- backward
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

struct BwdParams {
  int T, H, KV, Dq, Dkv, window;
  float scale_log2, scale;
  const float* lse;
  float* delta;                 // rowsum(dO * O): written by the dQ kernel, read by the dK/dV kernel
  const __nv_bfloat16* o;
  int64_t ldo;
  const __nv_bfloat16* dout;
  int64_t lddo;
  const __nv_bfloat16* qkv;  // the fused projection buffer (the dQ kernel reads its Q rows)
  int64_t ldqkv;
  __nv_bfloat16* dq;
  int64_t lddq;
  __nv_bfloat16* dk;
  int64_t lddk;
  __nv_bfloat16* dv;
  int64_t lddv;
  int* status;
};

// ---- dQ: one CTA per (128 queries, head, batch), 64-key blocks in a 6-stage K/V ring.
// TMEM: two S/dP sets (set s: S at [128s, +64), dP at [128s+64, +64)) so block j+1's scores are
// computed while the softmax warps turn block j into dS; dQ accumulates at [256, 384); the CTA's Q and
// dO rows sit at [384, 448) and [448, 512) as bf16 pairs, so the S and dP MMAs read only K and V from
// shared memory.
constexpr int BK64 = 64;
constexpr int KV64 = 64 * 128 * 2;        // 64 keys x 128 hd: two 8 KB swizzle atoms
constexpr int KV64_ATOM = 64 * 128;
constexpr int DQ_STAGES = 6;
constexpr int DQ_K = 0;                             // [6] x 16 KB
constexpr int DQ_V = DQ_K + DQ_STAGES * KV64;       // [6] x 16 KB
constexpr int DQ_DSUM = DQ_V + DQ_STAGES * KV64;    // [2][128] floats: half-row sums of dO * O
constexpr int DQ_BAR = DQ_DSUM + 1024;
constexpr int DQ_SMEM = DQ_BAR + 256 + 1024;
static_assert(DQ_SMEM <= 232448, "dQ kernel shared memory");

__global__ void __launch_bounds__(320, 1)
    attn_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, BwdParams p) {
  // tm_kv: 64-row boxes of the fused QKV buffer
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DQ_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                   // [DQ_STAGES]
  uint64_t* kv_empty = kv_full + DQ_STAGES;       // [DQ_STAGES]
  uint64_t* s_full = kv_empty + DQ_STAGES;        // [2]
  uint64_t* p_full = s_full + 2;                  // [2]: by iteration parity, so a warp group running one block ahead
                                  // arrives on the other barrier and never completes the current phase
  uint64_t* done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  static_assert((2 * DQ_STAGES + 7) * 8 <= 256, "dQ barrier region");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.H / p.KV);
  const int q0 = qb * BQ;
  const int w = p.window;
  const int kb_lo = max(0, q0 - w + 1) / BK64;
  const int kb_hi = min(q0 + BQ - 1, p.T - 1) / BK64;
  const int nkv = kb_hi - kb_lo + 1;
  const int warp = warp_id();
  if (device_failed(p.status)) return;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 256);  // every softmax thread has stored its Q or dO row in TMEM
    for (int i = 0; i < DQ_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 256);
    mbar_init(&p_full[1], 256);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) {
    *abort_flag = 1;
    if (p.status) atomicCAS(p.status, 0, code);
  };

  if (warp == 0) {
    if (elect_one()) {
      for (int j = 0; j < nkv; ++j) {
        const int st = j % DQ_STAGES;
        if (!mbar_wait(&kv_empty[st], ((j / DQ_STAGES) & 1) ^ 1, kBudgetNs, abort_flag, p.status)) {
          fail(kErrTimeoutProducer);
          break;
        }
        const int k0 = (kb_lo + j) * BK64;
        uint8_t* ks = smem + DQ_K + st * KV64;
        uint8_t* vs = smem + DQ_V + st * KV64;
        mbar_arrive_expect_tx(&kv_full[st], 2 * KV64);
        tma_load_3d(&tm_kv, &kv_full[st], ks, p.Dq + kvh * HD, k0, b);
        tma_load_3d(&tm_kv, &kv_full[st], ks + KV64_ATOM, p.Dq + kvh * HD + 64, k0, b);
        tma_load_3d(&tm_kv, &kv_full[st], vs, p.Dq + p.Dkv + kvh * HD, k0, b);
        tma_load_3d(&tm_kv, &kv_full[st], vs + KV64_ATOM, p.Dq + p.Dkv + kvh * HD + 64, k0, b);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 64, false, false);
      constexpr uint32_t idesc_q = umma_idesc_bf16(128, 128, false, true);
      bool ok = mbar_wait(q_full, 0, kBudgetNs, abort_flag, p.status);
      auto issue_sdp = [&](int j) -> bool {
        const int st = j % DQ_STAGES, set = j & 1;
        if (!mbar_wait(&kv_full[st], (j / DQ_STAGES) & 1, kBudgetNs, abort_flag, p.status)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + DQ_K + st * KV64), v_addr = smem_u32(smem + DQ_V + st * KV64);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t offb = (kk >> 2) * KV64_ATOM + (kk & 3) * 32;
          umma_bf16_ts(tmem + set * 128, tmem + 384 + kk * 8, umma_desc_sw128(k_addr + offb, 16, 1024), idesc_s,
                       kk > 0 ? 1u : 0u);
          umma_bf16_ts(tmem + set * 128 + 64, tmem + 448 + kk * 8, umma_desc_sw128(v_addr + offb, 16, 1024), idesc_s,
                       kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[set]);
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !issue_sdp(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = j % DQ_STAGES;
        const uint32_t k_addr = smem_u32(smem + DQ_K + st * KV64);
        // dS (bf16 pairs) sits in TMEM over the scores it came from: keys 32h .. 32h+31 at columns
        // 128*set + 32h .. +15, so each 16-key step reads its own 8 columns
#pragma unroll
        for (int kk = 0; kk < BK64 / 16; ++kk)
          umma_bf16_ts(tmem + 256, tmem + (j & 1) * 128 + (kk >> 1) * 32 + (kk & 1) * 8,
                       umma_desc_sw128(k_addr + kk * 2048, KV64_ATOM, 1024), idesc_q, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[st]);
      }
      if (!ok) fail(kErrTimeoutMma);
      umma_commit(done);
      mbar_wait(done, 0, kBudgetNs, nullptr);
    }
  } else {
    // 8 softmax warps: warps w and w+4 share TMEM lane group w%4 (rows) and split each block's columns
    const int wq = warp & 3, lane = lane_id();
    const int half = (warp - 2) >> 2;
    const int r = wq * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    const int qc = min(qi, p.T - 1);
    {
      // this row's Q (first warp of the row) or dO (second warp) into TMEM as bf16 pairs: the A operands
      // of the S and dP MMAs
      const int64_t m = (int64_t)b * p.T + qc;
      const uint4* src = reinterpret_cast<const uint4*>(half == 0 ? p.qkv + m * p.ldqkv + h * HD
                                                                  : p.dout + m * p.lddo + h * HD);
      uint32_t w0[32], w1[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 a = __ldg(src + i), c = __ldg(src + 8 + i);
        w0[4 * i] = a.x;
        w0[4 * i + 1] = a.y;
        w0[4 * i + 2] = a.z;
        w0[4 * i + 3] = a.w;
        w1[4 * i] = c.x;
        w1[4 * i + 1] = c.y;
        w1[4 * i + 2] = c.z;
        w1[4 * i + 3] = c.w;
      }
      tmem_st32(lane_base + 384 + 64 * half, w0);
      tmem_st32(lane_base + 384 + 64 * half + 32, w1);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(q_full);
    }
    const float lse2 = p.lse[((int64_t)b * p.H + h) * p.T + qc];  // log2 units
    // delta = rowsum(dO * O) over this head: the two warps of a row each reduce 64 of the 128 dims
    // (while the first tiles load) and meet in shared memory; the kernel writes delta for dK/dV
    float dl;
    {
      float* dsum = reinterpret_cast<float*>(smem + DQ_DSUM);
      const int64_t row = (int64_t)b * p.T + qc;
      const uint4* op = reinterpret_cast<const uint4*>(p.o + row * p.ldo + h * HD + half * 64);
      const uint4* gp = reinterpret_cast<const uint4*>(p.dout + row * p.lddo + h * HD + half * 64);
      uint4 ov[8], gv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ov[i] = __ldg(op + i);
        gv[i] = __ldg(gp + i);
      }
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t oa[4] = {ov[i].x, ov[i].y, ov[i].z, ov[i].w}, ga[4] = {gv[i].x, gv[i].y, gv[i].z, gv[i].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 x = unpack_bf16(oa[k]), y = unpack_bf16(ga[k]);
          acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
        }
      }
      dsum[half * 128 + r] = acc;
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
      dl = dsum[r] + dsum[128 + r];
      if (half == 0 && qi < p.T) p.delta[((int64_t)b * p.H + h) * p.T + qi] = dl;
    }
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int set = j & 1;
      if (!mbar_wait_warp(&s_full[set], (j >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
        fail(kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = (kb_lo + j) * BK64 + half * 32;
      const bool interior = (k0 + 31 <= q0) && (k0 > q0 + BQ - 1 - w) && (k0 + 32 <= p.T);
      uint32_t sv[32], dv[32];
      tmem_ld32(lane_base + set * 128 + half * 32, sv);
      tmem_ld32(lane_base + set * 128 + 64 + half * 32, dv);
      tmem_ld_wait();
      // dS = exp2(S * scale_log2 - lse2) (dP - delta); query qi sees key k0 + i for i in
      // [qi - w + 1 - k0, qi + 1 - k0) below T - k0 (boundary blocks only)
      uint32_t pk[16];
      auto body = [&](auto masked) {
        constexpr bool kMasked = decltype(masked)::value;
        uint32_t vis = 0xffffffffu;
        if constexpr (kMasked) vis = qi < p.T ? range_mask32(qi - w + 1 - k0, min(qi + 1 - k0, p.T - k0)) : 0u;
        const uint64_t dl2 = f32x2(dl, dl);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p0 = exp2f(fmaf(__uint_as_float(sv[i]), p.scale_log2, -lse2));
          float p1 = exp2f(fmaf(__uint_as_float(sv[i + 1]), p.scale_log2, -lse2));
          if constexpr (kMasked) {
            p0 = ((vis >> i) & 1u) ? p0 : 0.f;
            p1 = ((vis >> (i + 1)) & 1u) ? p1 : 0.f;
          }
          const float2 g = f32x2_split(
              mul_f32x2(f32x2(p0, p1), sub_f32x2(f32x2(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])), dl2)));
          pk[i / 2] = pack_bf16(g.x, g.y);
        }
      };
      if (interior) {
        body(std::false_type{});
      } else {
        body(std::true_type{});
      }
      // into this warp's own (already read) score columns: the other warp of the row still reads its half
      tmem_st16(lane_base + set * 128 + half * 32, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    if (ok && mbar_wait_warp(done, 0, kBudgetNs, abort_flag, p.status)) {
      tc_fence_after();
      __nv_bfloat16* row = p.dq + ((int64_t)b * p.T + qi) * p.lddq + h * HD;
#pragma unroll 1
      for (int c = half * 2; c < half * 2 + 2; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_base + 256 + c * 32, v);
        tmem_ld_wait();
        if (qi < p.T) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o;
            o.x = pack_bf16(__uint_as_float(v[8 * q + 0]) * p.scale, __uint_as_float(v[8 * q + 1]) * p.scale);
            o.y = pack_bf16(__uint_as_float(v[8 * q + 2]) * p.scale, __uint_as_float(v[8 * q + 3]) * p.scale);
            o.z = pack_bf16(__uint_as_float(v[8 * q + 4]) * p.scale, __uint_as_float(v[8 * q + 5]) * p.scale);
            o.w = pack_bf16(__uint_as_float(v[8 * q + 6]) * p.scale, __uint_as_float(v[8 * q + 7]) * p.scale);
            *reinterpret_cast<uint4*>(row + c * 32 + q * 8) = o;
          }
        }
      }
    } else if (ok) {
      fail(kErrTimeoutEpilogue);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- dK, dV: one CTA per (128 keys, kv head, batch), 64-query blocks in a 4-stage Q/dO ring.
// TMEM: two S^T/dP^T sets (set s: S^T at [128s, +64), dP^T at [128s+64, +64)), dV [256,384), dK [384,512).
constexpr int KB_Q = 64;
constexpr int HALF_TILE = 64 * 128 * 2;   // 64 rows x 128 hd, two 8 KB swizzle atoms
constexpr int HALF_ATOM = 64 * 128;
constexpr int DK_STAGES = 4;                        // Q/dO ring
constexpr int DK_K = 0;
constexpr int DK_V = DK_K + TILE_BYTES;
constexpr int DK_Q = DK_V + TILE_BYTES;            // [4] x HALF_TILE
constexpr int DK_DO = DK_Q + DK_STAGES * HALF_TILE;  // [4] x HALF_TILE
constexpr int DK_STAT = DK_DO + DK_STAGES * HALF_TILE; // [4] x (lse[64], delta[64]) floats
constexpr int DK_BAR = DK_STAT + DK_STAGES * 512;
constexpr int DK_SMEM = DK_BAR + 256 + 1024;
static_assert(DK_SMEM <= 232448, "dK/dV kernel shared memory");

__global__ void __launch_bounds__(320, 1)
    attn_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_qkv,
                        const __grid_constant__ CUtensorMap tm_do, BwdParams p) {
  // tm_kv: 128-row boxes (the CTA's K and V tiles); tm_qkv / tm_do: 64-row boxes (query blocks)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DK_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;                   // [DK_STAGES]
  uint64_t* qd_empty = qd_full + DK_STAGES;       // [DK_STAGES]
  uint64_t* s_full = qd_empty + DK_STAGES;        // [2]
  uint64_t* p_full = s_full + 2;                  // [2], by iteration parity (see the dQ kernel)
  uint64_t* done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  static_assert((2 * DK_STAGES + 7) * 8 <= 256, "dK/dV barrier region");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* stat = reinterpret_cast<float*>(smem + DK_STAT);

  const int kb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = p.H / p.KV;
  const int k0 = kb * BKV;
  const int w = p.window;
  const int qb_lo = k0 / KB_Q;
  const int qb_hi = min(p.T - 1, k0 + BKV - 1 + w - 1) / KB_Q;
  const int nq = qb_hi - qb_lo + 1;
  const int iters = nq * group;
  const int warp = warp_id();
  if (device_failed(p.status)) return;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < DK_STAGES; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 256);
    mbar_init(&p_full[1], 256);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) {
    *abort_flag = 1;
    if (p.status) atomicCAS(p.status, 0, code);
  };

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_3d(&tm_kv, kv_full, smem + DK_K, p.Dq + kvh * HD, k0, b);
      tma_load_3d(&tm_kv, kv_full, smem + DK_K + ATOM_BYTES, p.Dq + kvh * HD + 64, k0, b);
      tma_load_3d(&tm_kv, kv_full, smem + DK_V, p.Dq + p.Dkv + kvh * HD, k0, b);
      tma_load_3d(&tm_kv, kv_full, smem + DK_V + ATOM_BYTES, p.Dq + p.Dkv + kvh * HD + 64, k0, b);
      for (int it = 0; it < iters; ++it) {
        const int st = it % DK_STAGES;
        if (!mbar_wait(&qd_empty[st], ((it / DK_STAGES) & 1) ^ 1, kBudgetNs, abort_flag, p.status)) {
          fail(kErrTimeoutProducer);
          break;
        }
        const int h = kvh * group + it / nq;
        const int q0 = (qb_lo + it % nq) * KB_Q;
        uint8_t* qs = smem + DK_Q + st * HALF_TILE;
        uint8_t* ds = smem + DK_DO + st * HALF_TILE;
        float* ls = stat + st * 128;
        const int64_t srow = ((int64_t)b * p.H + h) * p.T + q0;
        mbar_arrive_expect_tx(&qd_full[st], 2 * HALF_TILE + 512);
        tma_load_3d(&tm_qkv, &qd_full[st], qs, h * HD, q0, b);
        tma_load_3d(&tm_qkv, &qd_full[st], qs + HALF_ATOM, h * HD + 64, q0, b);
        tma_load_3d(&tm_do, &qd_full[st], ds, h * HD, q0, b);
        tma_load_3d(&tm_do, &qd_full[st], ds + HALF_ATOM, h * HD + 64, q0, b);
        bulk_load(ls, p.lse + srow, 256, &qd_full[st]);
        bulk_load(ls + 64, p.delta + srow, 256, &qd_full[st]);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 64, false, false);
      constexpr uint32_t idesc_g = umma_idesc_bf16(128, 128, false, true);
      const uint32_t k_addr = smem_u32(smem + DK_K), v_addr = smem_u32(smem + DK_V);
      bool ok = mbar_wait(kv_full, 0, kBudgetNs, abort_flag, p.status);
      auto issue_s = [&](int it) -> bool {
        const int st = it % DK_STAGES, set = it & 1;
        if (!mbar_wait(&qd_full[st], (it / DK_STAGES) & 1, kBudgetNs, abort_flag, p.status)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + DK_Q + st * HALF_TILE);
        const uint32_t do_addr = smem_u32(smem + DK_DO + st * HALF_TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t offa = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
          const uint32_t offb = (kk >> 2) * HALF_ATOM + (kk & 3) * 32;
          umma_bf16_ss(tmem + set * 128, umma_desc_sw128(k_addr + offa, 16, 1024),
                       umma_desc_sw128(q_addr + offb, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          umma_bf16_ss(tmem + set * 128 + 64, umma_desc_sw128(v_addr + offa, 16, 1024),
                       umma_desc_sw128(do_addr + offb, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[set]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int it = 0; it < iters && ok; ++it) {
        if (it + 1 < iters && !issue_s(it + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&p_full[it & 1], (it >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = it % DK_STAGES, set = it & 1;
        const uint32_t q_addr = smem_u32(smem + DK_Q + st * HALF_TILE);
        const uint32_t do_addr = smem_u32(smem + DK_DO + st * HALF_TILE);
        // P^T and dS^T (bf16 pairs) sit in TMEM over S^T and dP^T: queries 32h .. 32h+31 at columns
        // 32h .. +15 of each, so each 16-query step reads its own 8 columns
#pragma unroll
        for (int kk = 0; kk < KB_Q / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          const uint32_t col = set * 128 + (kk >> 1) * 32 + (kk & 1) * 8;
          umma_bf16_ts(tmem + 256, tmem + col, umma_desc_sw128(do_addr + kk * 2048, HALF_ATOM, 1024), idesc_g, acc);
          umma_bf16_ts(tmem + 384, tmem + col + 64, umma_desc_sw128(q_addr + kk * 2048, HALF_ATOM, 1024), idesc_g,
                       acc);
        }
        umma_commit(&qd_empty[st]);
      }
      if (!ok) fail(kErrTimeoutMma);
      umma_commit(done);
      mbar_wait(done, 0, kBudgetNs, nullptr);
    }
  } else {
    // 8 softmax warps: warps w and w+4 share TMEM lane group w%4 (keys) and split each block's queries
    const int wq = warp & 3, lane = lane_id();
    const int half = (warp - 2) >> 2;
    const int r = wq * 32 + lane;
    const int kj = k0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    bool ok = true;
    for (int it = 0; it < iters; ++it) {
      const int set = it & 1, st = it % DK_STAGES;
      if (!mbar_wait_warp(&s_full[set], (it >> 1) & 1, kBudgetNs, abort_flag, p.status)) {
        fail(kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      const int q0 = (qb_lo + it % nq) * KB_Q + half * 32;
      const float* ls = stat + st * 128 + half * 32;
      // every (query, key) pair of these 32 queries visible to every key row of the tile
      const bool interior = (k0 + BKV - 1 <= q0) && (k0 > q0 + 31 - w) && (q0 + 32 <= p.T) && (k0 + BKV <= p.T);
      uint32_t sv[32], dv[32];
      tmem_ld32(lane_base + set * 128 + half * 32, sv);
      tmem_ld32(lane_base + set * 128 + 64 + half * 32, dv);
      tmem_ld_wait();
      // P^T = exp2(S^T * scale_log2 - lse2) and dS^T = P^T (dP^T - delta); key kj sees query q0 + i for
      // i in [kj - q0, kj - q0 + w) below T - q0 (boundary blocks only; interior blocks skip the mask)
      uint32_t pp[16], ss[16];
      auto body = [&](auto masked) {
        constexpr bool kMasked = decltype(masked)::value;
        uint32_t vis = 0xffffffffu;
        if constexpr (kMasked) vis = kj < p.T ? range_mask32(kj - q0, min(kj - q0 + w, p.T - q0)) : 0u;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(ls + i);
          const float4 d4 = *reinterpret_cast<const float4*>(ls + 64 + i);
          float pr[4];
          pr[0] = exp2f(fmaf(__uint_as_float(sv[i + 0]), p.scale_log2, -l4.x));
          pr[1] = exp2f(fmaf(__uint_as_float(sv[i + 1]), p.scale_log2, -l4.y));
          pr[2] = exp2f(fmaf(__uint_as_float(sv[i + 2]), p.scale_log2, -l4.z));
          pr[3] = exp2f(fmaf(__uint_as_float(sv[i + 3]), p.scale_log2, -l4.w));
          if constexpr (kMasked) {
#pragma unroll
            for (int k = 0; k < 4; ++k) pr[k] = ((vis >> (i + k)) & 1u) ? pr[k] : 0.f;
          }
          const float2 g0 = f32x2_split(mul_f32x2(
              f32x2(pr[0], pr[1]), sub_f32x2(f32x2(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])), f32x2(d4.x, d4.y))));
          const float2 g1 = f32x2_split(mul_f32x2(f32x2(pr[2], pr[3]), sub_f32x2(f32x2(__uint_as_float(dv[i + 2]),
                                                                                          __uint_as_float(dv[i + 3])),
                                                                                   f32x2(d4.z, d4.w))));
          pp[i / 2] = pack_bf16(pr[0], pr[1]);
          pp[i / 2 + 1] = pack_bf16(pr[2], pr[3]);
          ss[i / 2] = pack_bf16(g0.x, g0.y);
          ss[i / 2 + 1] = pack_bf16(g1.x, g1.y);
        }
      };
      if (interior) {
        body(std::false_type{});
      } else {
        body(std::true_type{});
      }
      // into this warp's own (already read) columns of S^T and dP^T
      tmem_st16(lane_base + set * 128 + half * 32, pp);
      tmem_st16(lane_base + set * 128 + 64 + half * 32, ss);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[it & 1]);
    }
    if (ok && mbar_wait_warp(done, 0, kBudgetNs, abort_flag, p.status)) {
      tc_fence_after();
      // half 0 writes dV, half 1 writes dK
      const bool isk = half == 1;
      __nv_bfloat16* row = isk ? p.dk + ((int64_t)b * p.T + kj) * p.lddk + kvh * HD
                               : p.dv + ((int64_t)b * p.T + kj) * p.lddv + kvh * HD;
      const float sc = isk ? p.scale : 1.f;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t v[32];
        tmem_ld32(lane_base + (isk ? 384 : 256) + cc * 32, v);
        tmem_ld_wait();
        if (kj < p.T) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o;
            o.x = pack_bf16(__uint_as_float(v[8 * q + 0]) * sc, __uint_as_float(v[8 * q + 1]) * sc);
            o.y = pack_bf16(__uint_as_float(v[8 * q + 2]) * sc, __uint_as_float(v[8 * q + 3]) * sc);
            o.z = pack_bf16(__uint_as_float(v[8 * q + 4]) * sc, __uint_as_float(v[8 * q + 5]) * sc);
            o.w = pack_bf16(__uint_as_float(v[8 * q + 6]) * sc, __uint_as_float(v[8 * q + 7]) * sc);
            *reinterpret_cast<uint4*>(row + cc * 32 + q * 8) = o;
          }
        }
      }
    } else if (ok) {
      fail(kErrTimeoutEpilogue);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// qkv: [B*T, Dq + 2*Dkv] bf16 (q | k | v columns, contiguous rows); o: [B*T, *] bf16 (head h at h*128).
void attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t T, int64_t H,
                 int64_t KV, int64_t hd, int64_t window) {
  TORCH_CHECK(hd == HD, "attn_fwd_tc: head_dim 128");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1, "attn_fwd_tc: bf16 rows");
  TORCH_CHECK(o.stride(1) == 1 && o.stride(0) % 8 == 0, "attn_fwd_tc: output rows");
  const int64_t W = qkv.size(1);
  TORCH_CHECK(W == (H + 2 * KV) * hd && H % KV == 0, "attn_fwd_tc: qkv width");
  c10::cuda::CUDAGuard g(qkv.device());
  CUtensorMap tm = tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.data_ptr(), W, T, B, qkv.stride(0),
                              qkv.stride(0) * T, 64, 128);
  FwdParams p;
  p.B = (int)B;
  p.T = (int)T;
  p.H = (int)H;
  p.KV = (int)KV;
  p.Dq = (int)(H * hd);
  p.Dkv = (int)(KV * hd);
  p.window = (int)std::min<int64_t>(window <= 0 ? T : window, T);
  p.scale_log2 = kLog2e / sqrtf((float)hd);
  p.out = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.status = status_ptr(qkv.device().index());
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM));
    attr = true;
  }
  // persistent: one CTA per SM (shared memory allows no more), no more CTAs than work items
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, qkv.device().index()));
  const int64_t items = ((T + 2 * BQ - 1) / (2 * BQ)) * H * B;
  attn_fwd_tc_kernel<<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(items, sms)), 320, FWD_SMEM,
                       at::cuda::getCurrentCUDAStream()>>>(tm, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br

namespace br {
// dqkv: [B*T, Dq + 2*Dkv] bf16 output (dq | dk | dv); dout: [B*T, H*hd] bf16; lse, delta: fp32 [B, H, T].
namespace {
void attn_bwd_tc_impl(const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout,
                      const torch::Tensor& lse, torch::Tensor& dqkv, torch::Tensor& delta, int64_t B, int64_t T,
                      int64_t H, int64_t KV, int64_t hd, int64_t window, int64_t which) {
  // which: 0 = dQ (which also writes delta) and dK/dV; 1 = dQ only; 2 = dK/dV only (delta already written)
  TORCH_CHECK(hd == HD && T % 128 == 0, "attn_bwd_tc: head_dim 128 and T % 128 == 0");
  const int64_t W = qkv.size(1);
  TORCH_CHECK(W == (H + 2 * KV) * hd && dqkv.size(1) == W, "attn_bwd_tc: widths");
  TORCH_CHECK(dout.stride(1) == 1 && dout.size(1) == H * hd, "attn_bwd_tc: dout");
  c10::cuda::CUDAGuard g(qkv.device());
  CUtensorMap tq = tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.data_ptr(), W, T, B, qkv.stride(0),
                              qkv.stride(0) * T, 64, 128);
  // the dK/dV kernel loads 64-query tiles of Q and dO
  CUtensorMap tq64 = tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.data_ptr(), W, T, B, qkv.stride(0),
                                qkv.stride(0) * T, 64, 64);
  CUtensorMap td64 = tma_map_3d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dout.data_ptr(), H * hd, T, B, dout.stride(0),
                                dout.stride(0) * T, 64, 64);
  BwdParams p;
  p.T = (int)T;
  p.H = (int)H;
  p.KV = (int)KV;
  p.Dq = (int)(H * hd);
  p.Dkv = (int)(KV * hd);
  p.window = (int)std::min<int64_t>(window <= 0 ? T : window, T);
  p.scale = 1.f / sqrtf((float)hd);
  p.scale_log2 = kLog2e * p.scale;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  TORCH_CHECK(o.stride(1) == 1 && o.stride(0) % 8 == 0 && dout.stride(0) % 8 == 0, "attn_bwd_tc: o / dout rows");
  p.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.lddo = dout.stride(0);
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ldqkv = qkv.stride(0);
  auto* base = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.dq = base;
  p.lddq = dqkv.stride(0);
  p.dk = base + H * hd;
  p.lddk = dqkv.stride(0);
  p.dv = base + (H + KV) * hd;
  p.lddv = dqkv.stride(0);
  p.status = status_ptr(qkv.device().index());
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DK_SMEM));
    attr = true;
  }
  auto st = at::cuda::getCurrentCUDAStream();
  if (which != 2) {
    attn_dq_tc_kernel<<<dim3((unsigned)(T / BQ), (unsigned)H, (unsigned)B), 320, DQ_SMEM, st>>>(tq64, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (which != 1) {
    attn_dkdv_tc_kernel<<<dim3((unsigned)(T / BKV), (unsigned)KV, (unsigned)B), 320, DK_SMEM, st>>>(tq, tq64, td64, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}
}  // namespace

void attn_bwd_tc(const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout, const torch::Tensor& lse,
                 torch::Tensor& dqkv, torch::Tensor& delta, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd,
                 int64_t window, int64_t which) {
  attn_bwd_tc_impl(qkv, o, dout, lse, dqkv, delta, B, T, H, KV, hd, window, which);
}

}  // namespace br
