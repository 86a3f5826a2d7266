// Causal sliding-window flash attention (head_dim 64 or 128, bf16 in, fp32 softmax), forward and backward.
//
// Semantics (src/model/gpt.ts:252-277): query i attends to keys j with i - w + 1 <= j <= i, where
// w is the layer's window (w >= T is plain causal); scores are scaled by 1/sqrt(hd). Key blocks
// entirely outside [i - w + 1, i] are skipped, so cost is O(T * w) instead of the reference's
// materialised [B, H, T, T] scores. The log-sum-exp per (b, h, t) is saved for the backward pass.
//
// Layout: q, k, v are column slices of the fused projection buffer [B*T, ld] (q at h*hd,
// k and v at their own offsets), o is [B*T, H*hd]; GQA maps head h to kv head h / (H/KV).
//
// Kernels (register-tiled warp MMAs, m16n8k16 bf16, ldmatrix from XOR-swizzled shared memory,
// cp.async double-buffered K/V tiles):
//   attn_fwd_kernel    128 queries per CTA (8 warps x 16 rows), 64-key blocks, online softmax.
//   attn_delta_kernel  delta = rowsum(dO * O).
//   attn_dq_kernel     64 queries per CTA: recompute P, dP = dO V^T, dS = P (dP - delta), dQ = dS K.
//   attn_dkdv_kernel   64 keys per CTA (4 warps x 16 keys): P^T, dV += P^T dO, dP^T = V dO^T,
//                      dK += dS^T Q; loops over the heads that share the kv head.
// The dQ and dK/dV passes each recompute the scores, which avoids fp32 atomics on dQ.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace br {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ldq, ldk, ldv;  // row strides (elements)
  int B, T, H, KV, window;
  float scale_log2;  // log2(e)/sqrt(hd)
};

__device__ __forceinline__ void cp_async16(uint32_t smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// byte offset of element (row, col) in a [rows][HD] bf16 tile with 16-byte chunks XOR-swizzled by row
// (HD / 8 >= 8 chunks per row, so the XOR with row & 7 stays inside the row)
template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return (uint32_t)(row * (2 * HD) + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1));
}

// Load `rows` rows (token index t0 + r of batch b) of a head slice into a swizzled tile.
template <int ROWS, int NTHREADS, int HD>
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16* base, int64_t ld, int b, int T, int t0,
                                          int col0) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
#pragma unroll
  for (int i = threadIdx.x; i < ROWS * CH; i += NTHREADS) {
    const int r = i / CH, c = i % CH;
    const int t = t0 + r;
    const bool ok = t < T && t >= 0;
    const __nv_bfloat16* g = base + ((int64_t)b * T + (ok ? t : 0)) * ld + col0 + c * 8;
    cp_async16(tile + swz<HD>(r, c * 8), g, ok);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16 rows x 16 k) at (r0, k0) of a swizzled tile, rows = M dim, cols = K dim.
template <int HD>
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], uint32_t tile, int r0, int k0) {
  const int l = threadIdx.x & 31;
  ldsm_x4(a, tile + swz<HD>(r0 + (l & 15), k0 + ((l >> 4) << 3)));
}
// B fragments for two n-tiles (16 n) x 16 k where the tile stores [n][k] (k contiguous).
template <int HD>
__device__ __forceinline__ void frag_b_nk(uint32_t (&b)[4], uint32_t tile, int n0, int k0) {
  const int l = threadIdx.x & 31;
  ldsm_x4(b, tile + swz<HD>(n0 + (l & 7) + ((l >> 4) << 3), k0 + (((l >> 3) & 1) << 3)));
}
// B fragments for two n-tiles (16 n) x 16 k where the tile stores [k][n] (n contiguous).
template <int HD>
__device__ __forceinline__ void frag_b_kn(uint32_t (&b)[4], uint32_t tile, int k0, int n0) {
  const int l = threadIdx.x & 31;
  ldsm_x4_t(b, tile + swz<HD>(k0 + (l & 7) + (((l >> 3) & 1) << 3), n0 + ((l >> 4) << 3)));
}
// Pack two accumulator n-tiles (16 rows x 16 cols) into an A fragment.
__device__ __forceinline__ void pack_a(uint32_t (&a)[4], const float (&c0)[4], const float (&c1)[4]) {
  a[0] = pack_bf16(c0[0], c0[1]);
  a[1] = pack_bf16(c0[2], c0[3]);
  a[2] = pack_bf16(c1[0], c1[1]);
  a[3] = pack_bf16(c1[2], c1[3]);
}

__device__ __forceinline__ bool visible(int qi, int kj, int T, int w) { return kj <= qi && kj > qi - w && kj < T; }

// ---------------------------------------------------------------------------------- forward
constexpr int F_BM = 128, F_BN = 64, F_THREADS = 256;
constexpr int f_smem(int HD) { return (F_BM + 2 * 2 * F_BN) * 2 * HD; }  // Q + double-buffered K, V

template <int HD>
__global__ void __launch_bounds__(F_THREADS, 2)
    attn_fwd_kernel(AttnArgs a, __nv_bfloat16* __restrict__ out, int64_t ldo, float* __restrict__ lse) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sQ = smem_u32(sm);
  const uint32_t sK = sQ + F_BM * 2 * HD;
  const uint32_t sV = sK + 2 * F_BN * 2 * HD;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.H / a.KV);
  const int q0 = qb * F_BM;
  const int w = a.window;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;

  const int kb_lo = max(0, q0 - w + 1) / F_BN;
  const int kb_hi = min(q0 + F_BM - 1, a.T - 1) / F_BN;

  load_tile<F_BM, F_THREADS, HD>(sQ, a.q, a.ldq, b, a.T, q0, h * HD);
  load_tile<F_BN, F_THREADS, HD>(sK, a.k, a.ldk, b, a.T, kb_lo * F_BN, kvh * HD);
  load_tile<F_BN, F_THREADS, HD>(sV, a.v, a.ldv, b, a.T, kb_lo * F_BN, kvh * HD);
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int r0 = warp * 16;
  const int qrow[2] = {q0 + r0 + g, q0 + r0 + g + 8};

  for (int kb = kb_lo; kb <= kb_hi; ++kb) {
    const int buf = (kb - kb_lo) & 1;
    if (kb < kb_hi) {
      load_tile<F_BN, F_THREADS, HD>(sK + (buf ^ 1) * F_BN * 2 * HD, a.k, a.ldk, b, a.T, (kb + 1) * F_BN, kvh * HD);
      load_tile<F_BN, F_THREADS, HD>(sV + (buf ^ 1) * F_BN * 2 * HD, a.v, a.ldv, b, a.T, (kb + 1) * F_BN, kvh * HD);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t tK = sK + buf * F_BN * 2 * HD, tV = sV + buf * F_BN * 2 * HD;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t af[4];
      frag_a<HD>(af, sQ, r0, kk * 16);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bf[4];
        frag_b_nk<HD>(bf, tK, np * 16, kk * 16);
        mma16816(s[2 * np], af, bf[0], bf[1]);
        mma16816(s[2 * np + 1], af, bf[2], bf[3]);
      }
    }
    const int k0 = kb * F_BN;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = k0 + nt * 8 + 2 * tq + (e & 1);
        const int ri = e >> 1;
        float x = s[nt][e] * a.scale_log2;
        if (!visible(qrow[ri], kj, a.T, w)) x = -INFINITY;
        s[nt][e] = x;
        mx[ri] = fmaxf(mx[ri], x);
      }
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffff, mx[ri], 1));
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffff, mx[ri], 2));
      const float mn = fmaxf(mrow[ri], mx[ri]);
      const float alpha = mn == -INFINITY ? 1.f : exp2f(mrow[ri] - mn);
      mrow[ri] = mn;
      lrow[ri] *= alpha;
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        o[i][2 * ri] *= alpha;
        o[i][2 * ri + 1] *= alpha;
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = e >> 1;
        const float p = mrow[ri] == -INFINITY ? 0.f : exp2f(s[nt][e] - mrow[ri]);
        s[nt][e] = p;
        lrow[ri] += p;
      }
#pragma unroll
    for (int kk = 0; kk < F_BN / 16; ++kk) {
      uint32_t af[4];
      pack_a(af, s[2 * kk], s[2 * kk + 1]);
#pragma unroll
      for (int nd = 0; nd < HD / 16; ++nd) {
        uint32_t bf[4];
        frag_b_kn<HD>(bf, tV, kk * 16, nd * 16);
        mma16816(o[2 * nd], af, bf[0], bf[1]);
        mma16816(o[2 * nd + 1], af, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    lrow[ri] += __shfl_xor_sync(0xffffffff, lrow[ri], 1);
    lrow[ri] += __shfl_xor_sync(0xffffffff, lrow[ri], 2);
  }
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int qi = qrow[ri];
    if (qi >= a.T) continue;
    const float inv = lrow[ri] > 0.f ? 1.f / lrow[ri] : 0.f;
    __nv_bfloat16* orow = out + ((int64_t)b * a.T + qi) * ldo + h * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt)
      *reinterpret_cast<uint32_t*>(orow + nt * 8 + 2 * tq) = pack_bf16(o[nt][2 * ri] * inv, o[nt][2 * ri + 1] * inv);
    if (tq == 0) lse[((int64_t)b * a.H + h) * a.T + qi] = (mrow[ri] + __log2f(lrow[ri])) / kLog2e;
  }
}

// ---------------------------------------------------------------------------------- delta
template <int HD>
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo, const __nv_bfloat16* __restrict__ dout,
                                  int64_t ldd, float* __restrict__ delta, int B, int T, int H) {
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)B * T * H;
  for (int64_t task = blockIdx.x * 8ll + (threadIdx.x >> 5); task < total; task += (int64_t)gridDim.x * 8) {
    const int h = (int)(task % H);
    const int64_t m = task / H;
    float s;
    if constexpr (HD == 128) {
      const uint2 ou = *reinterpret_cast<const uint2*>(o + m * ldo + h * HD + lane * 4);
      const uint2 du = *reinterpret_cast<const uint2*>(dout + m * ldd + h * HD + lane * 4);
      const float2 o0 = unpack_bf16(ou.x), o1 = unpack_bf16(ou.y), d0 = unpack_bf16(du.x), d1 = unpack_bf16(du.y);
      s = o0.x * d0.x + o0.y * d0.y + o1.x * d1.x + o1.y * d1.y;
    } else {
      const float2 o0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(o + m * ldo + h * HD + lane * 2));
      const float2 d0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(dout + m * ldd + h * HD + lane * 2));
      s = o0.x * d0.x + o0.y * d0.y;
    }
    s = warp_sum(s);
    const int b = (int)(m / T), t = (int)(m % T);
    if (lane == 0) delta[((int64_t)b * H + h) * T + t] = s;
  }
}

// ---------------------------------------------------------------------------------- dQ
constexpr int Q_BM = 64, Q_BN = 64, Q_THREADS = 128;
constexpr int q_smem(int HD) { return (2 * Q_BM + 2 * 2 * Q_BN) * 2 * HD; }  // Q, dO + double-buffered K, V

template <int HD>
__global__ void __launch_bounds__(Q_THREADS, 2)
    attn_dq_kernel(AttnArgs a, const __nv_bfloat16* __restrict__ dout, int64_t ldd, const float* __restrict__ lse,
                   const float* __restrict__ delta, __nv_bfloat16* __restrict__ dq, int64_t lddq) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sQ = smem_u32(sm);
  const uint32_t sdO = sQ + Q_BM * 2 * HD;
  const uint32_t sK = sdO + Q_BM * 2 * HD;
  const uint32_t sV = sK + 2 * Q_BN * 2 * HD;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.H / a.KV);
  const int q0 = qb * Q_BM;
  const int w = a.window;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int kb_lo = max(0, q0 - w + 1) / Q_BN;
  const int kb_hi = min(q0 + Q_BM - 1, a.T - 1) / Q_BN;

  load_tile<Q_BM, Q_THREADS, HD>(sQ, a.q, a.ldq, b, a.T, q0, h * HD);
  load_tile<Q_BM, Q_THREADS, HD>(sdO, dout, ldd, b, a.T, q0, h * HD);
  load_tile<Q_BN, Q_THREADS, HD>(sK, a.k, a.ldk, b, a.T, kb_lo * Q_BN, kvh * HD);
  load_tile<Q_BN, Q_THREADS, HD>(sV, a.v, a.ldv, b, a.T, kb_lo * Q_BN, kvh * HD);
  cp_async_commit();

  const int r0 = warp * 16;
  const int qrow[2] = {q0 + r0 + g, q0 + r0 + g + 8};
  float lse2[2], dl[2];
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int qi = min(qrow[ri], a.T - 1);
    lse2[ri] = lse[((int64_t)b * a.H + h) * a.T + qi] * kLog2e;
    dl[ri] = delta[((int64_t)b * a.H + h) * a.T + qi];
  }
  float acc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  for (int kb = kb_lo; kb <= kb_hi; ++kb) {
    const int buf = (kb - kb_lo) & 1;
    if (kb < kb_hi) {
      load_tile<Q_BN, Q_THREADS, HD>(sK + (buf ^ 1) * Q_BN * 2 * HD, a.k, a.ldk, b, a.T, (kb + 1) * Q_BN, kvh * HD);
      load_tile<Q_BN, Q_THREADS, HD>(sV + (buf ^ 1) * Q_BN * 2 * HD, a.v, a.ldv, b, a.T, (kb + 1) * Q_BN, kvh * HD);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t tK = sK + buf * Q_BN * 2 * HD, tV = sV + buf * Q_BN * 2 * HD;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t aq[4], ad[4];
      frag_a<HD>(aq, sQ, r0, kk * 16);
      frag_a<HD>(ad, sdO, r0, kk * 16);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bk[4], bv[4];
        frag_b_nk<HD>(bk, tK, np * 16, kk * 16);
        frag_b_nk<HD>(bv, tV, np * 16, kk * 16);
        mma16816(s[2 * np], aq, bk[0], bk[1]);
        mma16816(s[2 * np + 1], aq, bk[2], bk[3]);
        mma16816(dp[2 * np], ad, bv[0], bv[1]);
        mma16816(dp[2 * np + 1], ad, bv[2], bv[3]);
      }
    }
    const int k0 = kb * Q_BN;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = e >> 1;
        const int kj = k0 + nt * 8 + 2 * tq + (e & 1);
        const float p = visible(qrow[ri], kj, a.T, w) ? exp2f(s[nt][e] * a.scale_log2 - lse2[ri]) : 0.f;
        s[nt][e] = p * (dp[nt][e] - dl[ri]);
      }
#pragma unroll
    for (int kk = 0; kk < Q_BN / 16; ++kk) {
      uint32_t af[4];
      pack_a(af, s[2 * kk], s[2 * kk + 1]);
#pragma unroll
      for (int nd = 0; nd < HD / 16; ++nd) {
        uint32_t bf[4];
        frag_b_kn<HD>(bf, tK, kk * 16, nd * 16);
        mma16816(acc[2 * nd], af, bf[0], bf[1]);
        mma16816(acc[2 * nd + 1], af, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  const float sc = a.scale_log2 / kLog2e;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int qi = qrow[ri];
    if (qi >= a.T) continue;
    __nv_bfloat16* row = dq + ((int64_t)b * a.T + qi) * lddq + h * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt)
      *reinterpret_cast<uint32_t*>(row + nt * 8 + 2 * tq) = pack_bf16(acc[nt][2 * ri] * sc, acc[nt][2 * ri + 1] * sc);
  }
}

// ---------------------------------------------------------------------------------- dK, dV
constexpr int K_BN = 64, K_BM = 64, K_THREADS = 128;
constexpr int k_smem(int HD) { return (2 * K_BN + 2 * 2 * K_BM) * 2 * HD; }  // K, V + double-buffered Q, dO

template <int HD>
__global__ void __launch_bounds__(K_THREADS, 2)
    attn_dkdv_kernel(AttnArgs a, const __nv_bfloat16* __restrict__ dout, int64_t ldd, const float* __restrict__ lse,
                     const float* __restrict__ delta, __nv_bfloat16* __restrict__ dk, int64_t lddk,
                     __nv_bfloat16* __restrict__ dv, int64_t lddv) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sK = smem_u32(sm);
  const uint32_t sV = sK + K_BN * 2 * HD;
  const uint32_t sQ = sV + K_BN * 2 * HD;
  const uint32_t sdO = sQ + 2 * K_BM * 2 * HD;
  const int kb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = a.H / a.KV;
  const int k0 = kb * K_BN;
  const int w = a.window;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int qb_lo = k0 / K_BM;
  const int qb_hi = min(a.T - 1, k0 + K_BN - 1 + w - 1) / K_BM;
  const int nq = qb_hi - qb_lo + 1;

  load_tile<K_BN, K_THREADS, HD>(sK, a.k, a.ldk, b, a.T, k0, kvh * HD);
  load_tile<K_BN, K_THREADS, HD>(sV, a.v, a.ldv, b, a.T, k0, kvh * HD);
  const int r0 = warp * 16;
  const int krow[2] = {k0 + r0 + g, k0 + r0 + g + 8};
  float dka[HD / 8][4], dva[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dka[i][0] = dka[i][1] = dka[i][2] = dka[i][3] = dva[i][0] = dva[i][1] = dva[i][2] = dva[i][3] = 0.f;

  const int iters = nq * group;
  {
    const int h = kvh * group;
    load_tile<K_BM, K_THREADS, HD>(sQ, a.q, a.ldq, b, a.T, qb_lo * K_BM, h * HD);
    load_tile<K_BM, K_THREADS, HD>(sdO, dout, ldd, b, a.T, qb_lo * K_BM, h * HD);
    cp_async_commit();
  }
  for (int it = 0; it < iters; ++it) {
    const int buf = it & 1;
    const int h = kvh * group + it / nq;
    const int qb = qb_lo + it % nq;
    if (it + 1 < iters) {
      const int h2 = kvh * group + (it + 1) / nq, qb2 = qb_lo + (it + 1) % nq;
      load_tile<K_BM, K_THREADS, HD>(sQ + (buf ^ 1) * K_BM * 2 * HD, a.q, a.ldq, b, a.T, qb2 * K_BM, h2 * HD);
      load_tile<K_BM, K_THREADS, HD>(sdO + (buf ^ 1) * K_BM * 2 * HD, dout, ldd, b, a.T, qb2 * K_BM, h2 * HD);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t tQ = sQ + buf * K_BM * 2 * HD, tD = sdO + buf * K_BM * 2 * HD;
    const int q0 = qb * K_BM;
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t ak[4], av[4];
      frag_a<HD>(ak, sK, r0, kk * 16);
      frag_a<HD>(av, sV, r0, kk * 16);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bq[4], bd[4];
        frag_b_nk<HD>(bq, tQ, np * 16, kk * 16);
        frag_b_nk<HD>(bd, tD, np * 16, kk * 16);
        mma16816(st[2 * np], ak, bq[0], bq[1]);
        mma16816(st[2 * np + 1], ak, bq[2], bq[3]);
        mma16816(dpt[2 * np], av, bd[0], bd[1]);
        mma16816(dpt[2 * np + 1], av, bd[2], bd[3]);
      }
    }
    const float* lse_h = lse + ((int64_t)b * a.H + h) * a.T;
    const float* dl_h = delta + ((int64_t)b * a.H + h) * a.T;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int qa = q0 + nt * 8 + 2 * tq;
      const float l0 = qa < a.T ? lse_h[qa] * kLog2e : 0.f, l1 = qa + 1 < a.T ? lse_h[qa + 1] * kLog2e : 0.f;
      const float d0 = qa < a.T ? dl_h[qa] : 0.f, d1 = qa + 1 < a.T ? dl_h[qa + 1] : 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = e >> 1;
        const int qi = qa + (e & 1);
        const bool vis = visible(qi, krow[ri], a.T, w) && qi < a.T;
        const float p = vis ? exp2f(st[nt][e] * a.scale_log2 - ((e & 1) ? l1 : l0)) : 0.f;
        st[nt][e] = p;
        dpt[nt][e] = p * (dpt[nt][e] - ((e & 1) ? d1 : d0));
      }
    }
#pragma unroll
    for (int kk = 0; kk < K_BM / 16; ++kk) {
      uint32_t ap[4], as[4];
      pack_a(ap, st[2 * kk], st[2 * kk + 1]);
      pack_a(as, dpt[2 * kk], dpt[2 * kk + 1]);
#pragma unroll
      for (int nd = 0; nd < HD / 16; ++nd) {
        uint32_t bo[4], bq[4];
        frag_b_kn<HD>(bo, tD, kk * 16, nd * 16);
        frag_b_kn<HD>(bq, tQ, kk * 16, nd * 16);
        mma16816(dva[2 * nd], ap, bo[0], bo[1]);
        mma16816(dva[2 * nd + 1], ap, bo[2], bo[3]);
        mma16816(dka[2 * nd], as, bq[0], bq[1]);
        mma16816(dka[2 * nd + 1], as, bq[2], bq[3]);
      }
    }
    __syncthreads();
  }
  const float sc = a.scale_log2 / kLog2e;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int kj = krow[ri];
    if (kj >= a.T) continue;
    __nv_bfloat16* rk = dk + ((int64_t)b * a.T + kj) * lddk + kvh * HD;
    __nv_bfloat16* rv = dv + ((int64_t)b * a.T + kj) * lddv + kvh * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      *reinterpret_cast<uint32_t*>(rk + nt * 8 + 2 * tq) = pack_bf16(dka[nt][2 * ri] * sc, dka[nt][2 * ri + 1] * sc);
      *reinterpret_cast<uint32_t*>(rv + nt * 8 + 2 * tq) = pack_bf16(dva[nt][2 * ri], dva[nt][2 * ri + 1]);
    }
  }
}

AttnArgs make_args(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, int64_t B, int64_t T,
                   int64_t H, int64_t KV, int64_t hd, int64_t window) {
  TORCH_CHECK(hd == 64 || hd == 128, "attention kernels are built for head_dim 64 and 128");
  TORCH_CHECK(H % KV == 0, "H must be a multiple of KV");
  TORCH_CHECK(q.stride(1) == 1 && k.stride(1) == 1 && v.stride(1) == 1, "q/k/v rows must be contiguous");
  TORCH_CHECK(q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0, "row strides must be multiples of 8");
  AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.ldq = q.stride(0);
  a.ldk = k.stride(0);
  a.ldv = v.stride(0);
  a.B = (int)B;
  a.T = (int)T;
  a.H = (int)H;
  a.KV = (int)KV;
  a.window = (int)std::min<int64_t>(window <= 0 ? T : window, T);
  a.scale_log2 = kLog2e / sqrtf((float)hd);
  return a;
}

template <int HD>
void launch_fwd(const AttnArgs& a, torch::Tensor& o, torch::Tensor& lse) {
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, f_smem(HD)));
    attr = true;
  }
  dim3 grid((unsigned)((a.T + F_BM - 1) / F_BM), (unsigned)a.H, (unsigned)a.B);
  attn_fwd_kernel<HD><<<grid, F_THREADS, f_smem(HD), at::cuda::getCurrentCUDAStream()>>>(
      a, reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), o.stride(0), lse.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int HD>
void launch_delta(const torch::Tensor& o, const torch::Tensor& dout, torch::Tensor& delta, int64_t B, int64_t T,
                  int64_t H, cudaStream_t st) {
  const int64_t tasks = B * T * H;
  attn_delta_kernel<HD><<<(unsigned)std::min<int64_t>((tasks + 7) / 8, 148 * 16), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), o.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0), delta.data_ptr<float>(), (int)B, (int)T,
      (int)H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int HD>
void launch_bwd(const AttnArgs& a, const torch::Tensor& o, const torch::Tensor& dout, const torch::Tensor& lse,
                torch::Tensor& dq, torch::Tensor& dk, torch::Tensor& dv, torch::Tensor& delta) {
  auto st = at::cuda::getCurrentCUDAStream();
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, q_smem(HD)));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, k_smem(HD)));
    attr = true;
  }
  launch_delta<HD>(o, dout, delta, a.B, a.T, a.H, st);
  attn_dq_kernel<HD><<<dim3((unsigned)((a.T + Q_BM - 1) / Q_BM), (unsigned)a.H, (unsigned)a.B), Q_THREADS, q_smem(HD),
                       st>>>(a, reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
                             lse.data_ptr<float>(), delta.data_ptr<float>(),
                             reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), dq.stride(0));
  attn_dkdv_kernel<HD><<<dim3((unsigned)((a.T + K_BN - 1) / K_BN), (unsigned)a.KV, (unsigned)a.B), K_THREADS,
                         k_smem(HD), st>>>(a, reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
                                           lse.data_ptr<float>(), delta.data_ptr<float>(),
                                           reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()), dk.stride(0),
                                           reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), dv.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// q, k, v: [B*T, *] column slices (head h at h*hd); o: [B*T, H*hd]; lse: fp32 [B, H, T]. hd: 64 or 128.
void attn_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& o,
              torch::Tensor& lse, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd, int64_t window) {
  AttnArgs a = make_args(q, k, v, B, T, H, KV, hd, window);
  c10::cuda::CUDAGuard guard(q.device());
  if (hd == 128)
    launch_fwd<128>(a, o, lse);
  else
    launch_fwd<64>(a, o, lse);
}

// dq, dk, dv: column slices like q, k, v (may live in one fused [B*T, 3D] buffer).
void attn_bwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& o,
              const torch::Tensor& dout, const torch::Tensor& lse, torch::Tensor& dq, torch::Tensor& dk,
              torch::Tensor& dv, torch::Tensor& delta, torch::Tensor& dq_acc, int64_t B, int64_t T, int64_t H,
              int64_t KV, int64_t hd, int64_t window) {
  (void)dq_acc;
  AttnArgs a = make_args(q, k, v, B, T, H, KV, hd, window);
  c10::cuda::CUDAGuard guard(q.device());
  if (hd == 128)
    launch_bwd<128>(a, o, dout, lse, dq, dk, dv, delta);
  else
    launch_bwd<64>(a, o, dout, lse, dq, dk, dv, delta);
}

}  // namespace br
