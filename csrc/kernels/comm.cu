// In-kernel data-parallel collectives over NVLink / NVSwitch peer memory.
//
// Symmetric buffers: each rank cudaMallocs a region, exports a CUDA IPC handle, and opens its peers'
// handles (peer access is enabled lazily by the driver); kernels then read peers' memory with plain
// loads. No multicast, no TMA on peer memory.
//
// Step protocol (epoch = training step, monotonic):
//   pack      local fp32 gradients of a bucket -> this rank's symmetric send buffer in the wire
//             dtype (fp32 / bf16 / fp16), fused with a non-finite check;
//   signal    flags[slot] = epoch with a system-scope release store (separate 1-thread launch after
//             the pack kernel on the same stream, so all of the bucket is written first);
//   reduce    for every element of the segments this rank owns inside the bucket: wait (acquire,
//             bounded) until every peer's flags[slot] >= epoch, then out = scale * sum_p send_p;
//   push      after its optimizer step, each owner writes its parameters into every peer's symmetric
//             parameter buffer with posted stores and release-stores its slot of each peer's
//             push-flag array; a receiver acquires its local flags, then refreshes the bf16 GEMM
//             shadows of the parameters it does not own (the training path);
//   gather    the pull form of the same exchange: each rank reads the parameters it does not own from
//             the owners' buffers after an acquire on the owner's flag (remote loads pay a round trip
//             each, which caps them well below the stores' bandwidth at 8 ranks).
// A wait that exceeds its budget records kErrTimeoutPeer in the device status word and the block
// skips its work; the host treats the step as aborted (the reference's abort-and-skip), so nothing
// spins forever and nothing traps.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cuda_fp16.h>

#include "common.cuh"
#include "status.h"

namespace br {
namespace {

enum Wire : int { W_F32 = 0, W_BF16 = 1, W_F16 = 2 };

__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Waits (thread 0 of the block) until flags_p[slot] >= epoch for every peer; returns false on timeout.
__device__ bool wait_peers(const int64_t* const* flags, int npeers, int slot, int64_t epoch, uint64_t budget_ns,
                           int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < npeers && ok; ++p) {
      const int64_t* f = flags[p] + slot;
      uint32_t it = 0;
      while (ld_acquire_sys(f) < epoch) {
        if ((++it & 63u) == 0 && globaltimer_ns() - t0 > budget_ns) {
          ok = 0;
          if (status) atomicCAS(status, 0, kErrTimeoutPeer);
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

struct Chunk {
  int64_t off;
  int64_t len;
};

template <int WIRE>
__device__ __forceinline__ void load8(const void* base, int64_t i, float (&v)[8]) {
  // peers' buffers are read with L2-only loads (.cg): L1 is not coherent with another GPU's writes
  if constexpr (WIRE == W_F32) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + i));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (WIRE == W_BF16) {
        const float2 f = unpack_bf16(w[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
        const float2 f = __half22float2(h);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      }
    }
  }
}

template <int WIRE>
__device__ __forceinline__ float load1(const void* base, int64_t i) {
  if constexpr (WIRE == W_F32) return __ldcg(reinterpret_cast<const float*>(base) + i);
  const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(base) + i);
  if constexpr (WIRE == W_BF16) return __bfloat162float(__ushort_as_bfloat16(u));
  return __half2float(__ushort_as_half(u));
}

template <int WIRE>
__device__ __forceinline__ void store_wire(void* base, int64_t i, float x) {
  if constexpr (WIRE == W_F32) reinterpret_cast<float*>(base)[i] = x;
  else if constexpr (WIRE == W_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16(x);
  else reinterpret_cast<__half*>(base)[i] = __float2half(x);
}

template <int WIRE>
__device__ __forceinline__ void store_wire4(void* base, int64_t i, float4 x) {
  if constexpr (WIRE == W_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i) = x;
  } else if constexpr (WIRE == W_BF16) {
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(base) + i) = make_uint2(pack_bf16(x.x, x.y), pack_bf16(x.z, x.w));
  } else {
    const __half2 a = __floats2half2_rn(x.x, x.y), b = __floats2half2_rn(x.z, x.w);
    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(base) + i) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
}

// grid-stride over [lo, hi): send[i] = wire(src[i] * scale); *bad |= any non-finite. The 4-aligned body
// moves 16-byte loads and 8/16-byte stores; the unaligned head and tail go element by element.
template <int WIRE>
__global__ void pack_kernel(const float* __restrict__ src, void* __restrict__ send, int64_t lo, int64_t hi, float scale,
                            int* __restrict__ bad) {
  int nonfinite = 0;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t a = min(hi, (lo + 3) & ~int64_t(3));
  const int64_t b4 = a + ((hi - a) & ~int64_t(3));
  for (int64_t i = lo + tid; i < a; i += nth) {
    const float x = src[i] * scale;
    nonfinite |= !isfinite(x);
    store_wire<WIRE>(send, i, x);
  }
  for (int64_t i = a + tid * 4; i < b4; i += nth * 4) {
    float4 x = *reinterpret_cast<const float4*>(src + i);
    x.x *= scale;
    x.y *= scale;
    x.z *= scale;
    x.w *= scale;
    nonfinite |= !(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w));
    store_wire4<WIRE>(send, i, x);
  }
  for (int64_t i = b4 + tid; i < hi; i += nth) {
    const float x = src[i] * scale;
    nonfinite |= !isfinite(x);
    store_wire<WIRE>(send, i, x);
  }
  if (__syncthreads_or(nonfinite) && threadIdx.x == 0) atomicOr(bad, 1);
}

__global__ void signal_kernel(int64_t* flag, int64_t value) {
  __threadfence_system();
  st_release_sys(flag, value);
}

// One block per chunk (grid-stride over chunks). out[i] = scale * sum_p send_p[i], summed in peer order
// (the same order on every owner, so results are deterministic). Each thread keeps kRedUnroll 16-byte
// loads per peer in flight to cover NVLink latency.
constexpr int kRedUnroll = 4;

template <int WIRE>
__global__ void __launch_bounds__(256) reduce_kernel(const void* const* __restrict__ peers, const int64_t* const* flags,
                                                     int npeers, int slot, int64_t epoch, const Chunk* __restrict__ chunks,
                                                     int nchunks, float* __restrict__ out, float scale,
                                                     uint64_t budget_ns, int* status) {
  if (!wait_peers(flags, npeers, slot, epoch, budget_ns, status)) return;
  const int64_t step = (int64_t)blockDim.x * 8;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const Chunk ch = chunks[c];
    const int64_t n8 = ch.len & ~int64_t(7);
    int64_t j = threadIdx.x * 8;
    for (; j + (kRedUnroll - 1) * step < n8; j += kRedUnroll * step) {
      float acc[kRedUnroll][8];
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[u][k] = 0.f;
      for (int p = 0; p < npeers; ++p) {
        float v[kRedUnroll][8];
#pragma unroll
        for (int u = 0; u < kRedUnroll; ++u) load8<WIRE>(peers[p], ch.off + j + u * step, v[u]);
#pragma unroll
        for (int u = 0; u < kRedUnroll; ++u)
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[u][k] += v[u][k];
      }
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u) {
        float4* o = reinterpret_cast<float4*>(out + ch.off + j + u * step);
        o[0] = make_float4(acc[u][0] * scale, acc[u][1] * scale, acc[u][2] * scale, acc[u][3] * scale);
        o[1] = make_float4(acc[u][4] * scale, acc[u][5] * scale, acc[u][6] * scale, acc[u][7] * scale);
      }
    }
    for (; j < n8; j += step) {
      const int64_t i = ch.off + j;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int p = 0; p < npeers; ++p) {
        float v[8];
        load8<WIRE>(peers[p], i, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += v[k];
      }
      float4* o = reinterpret_cast<float4*>(out + i);
      o[0] = make_float4(acc[0] * scale, acc[1] * scale, acc[2] * scale, acc[3] * scale);
      o[1] = make_float4(acc[4] * scale, acc[5] * scale, acc[6] * scale, acc[7] * scale);
    }
    for (int64_t jj = n8 + threadIdx.x; jj < ch.len; jj += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < npeers; ++p) acc += load1<WIRE>(peers[p], ch.off + jj);
      out[ch.off + jj] = acc * scale;
    }
  }
}

struct GatherSeg {
  int64_t off;        // element offset in the flat parameter buffer
  int64_t len;
  int64_t owner;
  int64_t cols;       // shadow row length (elements); 0 when no shadow
  int64_t shadow_ld;
  int64_t shadow;     // bf16 shadow base pointer of the parameter, 0 if none
  int64_t start;      // element offset of this chunk inside its parameter (for shadow row/col)
};

__global__ void __launch_bounds__(256) gather_kernel(const float* const* __restrict__ peers, const int64_t* const* flags,
                                                     int npeers, int slot, int64_t epoch,
                                                     const GatherSeg* __restrict__ segs, int nsegs,
                                                     float* __restrict__ local, uint64_t budget_ns, int* status) {
  if (!wait_peers(flags, npeers, slot, epoch, budget_ns, status)) return;
  constexpr int U = 4;
  for (int s = blockIdx.x; s < nsegs; s += gridDim.x) {
    const GatherSeg g = segs[s];
    const float* src = peers[g.owner] + g.off;
    float* dst = local + g.off;
    __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(g.shadow);
    // 4 consecutive elements stay in one shadow row when the row length, the leading dimension and
    // the chunk start are multiples of 4
    const bool vec = (g.off & 3) == 0 && (g.start & 3) == 0 &&
                     (!sh || ((g.cols & 3) == 0 && (g.shadow_ld & 3) == 0 && (g.shadow & 7) == 0));
    const int64_t n4 = vec ? (g.len & ~int64_t(3)) : 0;
    const int64_t step = (int64_t)blockDim.x * 4;
    for (int64_t j0 = threadIdx.x * 4; j0 < n4; j0 += U * step) {
      float4 x[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = j0 + u * step;
        if (j < n4) x[u] = __ldcg(reinterpret_cast<const float4*>(src + j));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = j0 + u * step;
        if (j < n4) {
          *reinterpret_cast<float4*>(dst + j) = x[u];
          if (sh) {
            const int64_t e = g.start + j;
            *reinterpret_cast<uint2*>(sh + (e / g.cols) * g.shadow_ld + (e % g.cols)) =
                make_uint2(pack_bf16(x[u].x, x[u].y), pack_bf16(x[u].z, x[u].w));
          }
        }
      }
    }
    for (int64_t j = n4 + threadIdx.x; j < g.len; j += blockDim.x) {
      const float x = __ldcg(src + j);
      dst[j] = x;
      if (sh) {
        const int64_t e = g.start + j;
        sh[(e / g.cols) * g.shadow_ld + (e % g.cols)] = __float2bfloat16(x);
      }
    }
  }
}

// ------------------------------------------------------------------------------ parameter push
// The owner of each parameter writes its updated values into every peer's symmetric parameter buffer
// (posted NVLink stores: no round trip per load, unlike a pull), then stores `epoch` into its slot of
// each peer's push-flag array. A receiver waits on its own (local) flag slots, then refreshes the bf16
// GEMM shadows of the parameters it does not own from local memory.

// grid-stride over owned chunks: peers[p][off + j] = src[off + j] for every peer p != me
__global__ void __launch_bounds__(256) push_kernel(const float* __restrict__ src, float* const* __restrict__ peers,
                                                   int npeers, int me, const Chunk* __restrict__ chunks, int nchunks) {
  constexpr int U = 4;
  const int64_t step = (int64_t)blockDim.x * 4;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const Chunk ch = chunks[c];
    const float* s = src + ch.off;
    const int64_t n4 = ch.len & ~int64_t(3);
    for (int64_t j0 = threadIdx.x * 4; j0 < n4; j0 += U * step) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = j0 + u * step;
        if (j < n4) v[u] = *reinterpret_cast<const float4*>(s + j);
      }
      // peers in order from me + 1, so the ranks start on different peers
      for (int k = 1; k < npeers; ++k) {
        const int p = me + k < npeers ? me + k : me + k - npeers;
        float* d = peers[p] + ch.off;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + u * step;
          if (j < n4) *reinterpret_cast<float4*>(d + j) = v[u];
        }
      }
    }
    for (int64_t j = n4 + threadIdx.x; j < ch.len; j += blockDim.x) {
      const float x = s[j];
      for (int k = 1; k < npeers; ++k) peers[me + k < npeers ? me + k : me + k - npeers][ch.off + j] = x;
    }
  }
}

// flags[p][me] = epoch on every peer p != me, after this GPU's earlier writes (release, system scope)
__global__ void signal_peers_kernel(int64_t* const* flags, int npeers, int me, int64_t epoch) {
  __threadfence_system();
  for (int p = 0; p < npeers; ++p)
    if (p != me) st_release_sys(flags[p] + me, epoch);
}

// Every block first waits (bounded) until each other rank's slot of this rank's push-flag array holds
// `epoch`, then writes the bf16 shadows of the listed (non-owned) segments from the local fp32 values.
__global__ void __launch_bounds__(256) shadow_refresh_kernel(const float* __restrict__ params,
                                                             const int64_t* __restrict__ push_flags, int npeers,
                                                             int me, int64_t epoch,
                                                             const GatherSeg* __restrict__ segs, int nsegs,
                                                             uint64_t budget_ns, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < npeers && ok; ++p) {
      if (p == me) continue;
      uint32_t it = 0;
      while (ld_acquire_sys(push_flags + p) < epoch) {
        if ((++it & 63u) == 0 && globaltimer_ns() - t0 > budget_ns) {
          ok = 0;
          if (status) atomicCAS(status, 0, kErrTimeoutPeer);
          break;
        }
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  for (int s = blockIdx.x; s < nsegs; s += gridDim.x) {
    const GatherSeg g = segs[s];
    if (!g.shadow) continue;
    const float* src = params + g.off;
    __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(g.shadow);
    const bool vec = (g.off & 3) == 0 && (g.start & 3) == 0 && (g.cols & 3) == 0 && (g.shadow_ld & 3) == 0 &&
                     (g.shadow & 7) == 0;
    const int64_t n4 = vec ? (g.len & ~int64_t(3)) : 0;
    for (int64_t j = threadIdx.x * 4; j < n4; j += (int64_t)blockDim.x * 4) {
      const float4 x = *reinterpret_cast<const float4*>(src + j);
      const int64_t e = g.start + j;
      *reinterpret_cast<uint2*>(sh + (e / g.cols) * g.shadow_ld + (e % g.cols)) =
          make_uint2(pack_bf16(x.x, x.y), pack_bf16(x.z, x.w));
    }
    for (int64_t j = n4 + threadIdx.x; j < g.len; j += blockDim.x) {
      const int64_t e = g.start + j;
      sh[(e / g.cols) * g.shadow_ld + (e % g.cols)] = __float2bfloat16(src[j]);
    }
  }
}

// ------------------------------------------------------------------------------ push reduce-scatter
// The gradient reduce-scatter the trainer runs. Every rank packs a finished bucket into the wire dtype and
// stores each parameter's slice straight into its owner's receive buffer, in the slot of the sending rank
// (posted NVLink stores for peers: no load ever crosses the link); a one-thread kernel then release-stores
// (2 * epoch + this rank's non-finite bit) into flags[bucket][me] of every rank. Each owner waits on its
// own (local) flags and sums the N slots from local memory in rank order (deterministic), scaled by 1/N.
// Receive layout on rank o: [source rank][slot_elems] in the wire dtype, parameters at their offsets in
// o's owned space. The non-finite bits of the last bucket's flags give every rank the same skip decision.

struct PushChunk {
  int64_t off;       // element offset in the flat gradient buffer
  int64_t len;
  int64_t owner;
  int64_t slot_off;  // element offset inside the owner's per-source slot
};

template <int WIRE>
__device__ __forceinline__ void store_wire8(void* base, int64_t i, const float (&x)[8]) {
  if constexpr (WIRE == W_F32) {
    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i);
    d[0] = make_float4(x[0], x[1], x[2], x[3]);
    d[1] = make_float4(x[4], x[5], x[6], x[7]);
  } else if constexpr (WIRE == W_BF16) {
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + i) =
        make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
  } else {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __half2 h = __floats2half2_rn(x[2 * k], x[2 * k + 1]);
      w[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(base) + i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

constexpr int kPushUnroll = 4;

// grid-stride over the bucket's chunks: recv[owner][me * slot + slot_off + j] = wire(grad[off + j] * scale)
template <int WIRE>
__global__ void __launch_bounds__(256) pack_push_kernel(const float* __restrict__ grad, void* const* __restrict__ recv,
                                                        int me, int64_t slot_elems,
                                                        const PushChunk* __restrict__ chunks, int nchunks,
                                                        float scale, int* __restrict__ bad) {
  int nonfinite = 0;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const PushChunk ch = chunks[c];
    const float* src = grad + ch.off;
    void* dst = recv[ch.owner];
    const int64_t base = (int64_t)me * slot_elems + ch.slot_off;
    const int64_t n8 = ch.len & ~int64_t(7);
    const int64_t step = (int64_t)blockDim.x * 8;
    // kPushUnroll independent 32-byte loads per thread in flight (the kernel is latency-bound otherwise)
    for (int64_t j0 = threadIdx.x * 8; j0 < n8; j0 += kPushUnroll * step) {
      float4 a[kPushUnroll], b[kPushUnroll];
#pragma unroll
      for (int u = 0; u < kPushUnroll; ++u) {
        const int64_t j = j0 + u * step;
        if (j < n8) {
          a[u] = __ldcs(reinterpret_cast<const float4*>(src + j));
          b[u] = __ldcs(reinterpret_cast<const float4*>(src + j + 4));
        }
      }
#pragma unroll
      for (int u = 0; u < kPushUnroll; ++u) {
        const int64_t j = j0 + u * step;
        if (j < n8) {
          float x[8] = {a[u].x * scale, a[u].y * scale, a[u].z * scale, a[u].w * scale,
                        b[u].x * scale, b[u].y * scale, b[u].z * scale, b[u].w * scale};
#pragma unroll
          for (int k = 0; k < 8; ++k) nonfinite |= !isfinite(x[k]);
          store_wire8<WIRE>(dst, base + j, x);
        }
      }
    }
    for (int64_t j = n8 + threadIdx.x; j < ch.len; j += blockDim.x) {
      const float x = src[j] * scale;
      nonfinite |= !isfinite(x);
      store_wire<WIRE>(dst, base + j, x);
    }
  }
  if (__syncthreads_or(nonfinite) && threadIdx.x == 0) atomicOr(bad, 1);
}

// flags[p][slot * npeers + me] = 2 * epoch + (bad != 0) on every rank p (this one included), after all of
// this GPU's earlier writes (release, system scope)
__global__ void signal_all_kernel(int64_t* const* flags, int npeers, int me, int slot, int64_t epoch,
                                  const int* bad) {
  __threadfence_system();
  const int64_t v = 2 * epoch + (*bad ? 1 : 0);
  for (int p = 0; p < npeers; ++p) st_release_sys(flags[p] + (int64_t)slot * npeers + me, v);
}

// Waits (thread 0, bounded) until every source's flag of `slot` in this rank's (local) flag array has
// reached 2 * epoch; returns false on timeout. The result reaches the block through __syncthreads_and, so
// the kernel needs no shared memory and can share an SM with a kernel that fills it.
__device__ bool wait_local_flags(const int64_t* flags, int npeers, int slot, int64_t epoch, uint64_t budget_ns,
                                 int* status) {
  int ok = 1;
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    const int64_t* f = flags + (int64_t)slot * npeers;
    for (int p = 0; p < npeers && ok; ++p) {
      uint32_t it = 0;
      while (ld_acquire_sys(f + p) < 2 * epoch) {
        if ((++it & 63u) == 0 && globaltimer_ns() - t0 > budget_ns) {
          ok = 0;
          if (status) atomicCAS(status, 0, kErrTimeoutPeer);
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// out[off + j] = scale * sum over sources (in rank order) of recv[src * slot + slot_off + j], for the chunks
// of the bucket this rank owns; all reads are local.
template <int WIRE>
__global__ void __launch_bounds__(256) reduce_local_kernel(const void* __restrict__ recv, const int64_t* flags,
                                                           int npeers, int slot, int64_t epoch, int64_t slot_elems,
                                                           const PushChunk* __restrict__ chunks, int nchunks,
                                                           float* __restrict__ out, float scale, uint64_t budget_ns,
                                                           int* status) {
  if (!wait_local_flags(flags, npeers, slot, epoch, budget_ns, status)) return;
  const int64_t step = (int64_t)blockDim.x * 8;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const PushChunk ch = chunks[c];
    const int64_t n8 = ch.len & ~int64_t(7);
    // kRedUnroll independent 16-byte loads per source in flight per thread
    for (int64_t j0 = threadIdx.x * 8; j0 < n8; j0 += kRedUnroll * step) {
      float acc[kRedUnroll][8];
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[u][k] = 0.f;
      for (int p = 0; p < npeers; ++p) {
        float v[kRedUnroll][8];
#pragma unroll
        for (int u = 0; u < kRedUnroll; ++u)
          if (j0 + u * step < n8) load8<WIRE>(recv, (int64_t)p * slot_elems + ch.slot_off + j0 + u * step, v[u]);
#pragma unroll
        for (int u = 0; u < kRedUnroll; ++u)
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[u][k] += v[u][k];
      }
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u) {
        const int64_t j = j0 + u * step;
        if (j < n8) {
          float4* o = reinterpret_cast<float4*>(out + ch.off + j);
          o[0] = make_float4(acc[u][0] * scale, acc[u][1] * scale, acc[u][2] * scale, acc[u][3] * scale);
          o[1] = make_float4(acc[u][4] * scale, acc[u][5] * scale, acc[u][6] * scale, acc[u][7] * scale);
        }
      }
    }
    for (int64_t j = n8 + threadIdx.x; j < ch.len; j += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < npeers; ++p) acc += load1<WIRE>(recv, (int64_t)p * slot_elems + ch.slot_off + j);
      out[ch.off + j] = acc * scale;
    }
  }
}

// One thread: waits for every source's flag of `slot` (the step's last bucket), then
// skip = OR of their non-finite bits, or 1 when a wait timed out or a kernel reported an error this step.
__global__ void agree_kernel(const int64_t* flags, int npeers, int slot, int64_t epoch, int* skip,
                             uint64_t budget_ns, int* status) {
  const uint64_t t0 = globaltimer_ns();
  const int64_t* f = flags + (int64_t)slot * npeers;
  int any = 0;
  for (int p = 0; p < npeers; ++p) {
    uint32_t it = 0;
    int64_t v;
    while ((v = ld_acquire_sys(f + p)) < 2 * epoch) {
      if ((++it & 63u) == 0 && globaltimer_ns() - t0 > budget_ns) {
        atomicCAS(status, 0, kErrTimeoutPeer);
        v = 2 * epoch + 1;
        break;
      }
    }
    any |= (int)(v & 1);
  }
  *skip = (any || *reinterpret_cast<volatile int*>(status) != 0) ? 1 : 0;
}

// ------------------------------------------------------------------------------ top-k + error feedback
// Deep Gradient Compression as in the reference sparsifier (gradient-sparsifier.ts:82-144), per bucket:
//   g = grad * scale + e (+ momentum correction v = mu*v + g, g = v); thr = the floor(S*(1-k))-th
//   smallest of S sampled |g|; keep |g| >= thr (e = 0) else e = g. Kept entries go on the wire as
//   (u32 index, f16 value) pairs, appended to the list of the element's owner.
// masking != 0 (with a velocity) runs the published form instead: u = mu*u + grad*scale, g = e + u,
// and both e and u are cleared where the entry is sent.

__device__ __forceinline__ uint32_t hash_u32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

// One block: sample, sort (bitonic in shared memory) and pick the threshold for bucket [lo, hi).
__global__ void __launch_bounds__(1024) topk_threshold_kernel(const float* __restrict__ grad, const float* __restrict__ err,
                                                              const float* __restrict__ vel, int64_t lo, int64_t hi,
                                                              float scale, float mu, int S, float keep_ratio,
                                                              uint32_t seed, int masking, float* __restrict__ thr_out) {
  extern __shared__ float smp[];  // S (power of two)
  const int64_t n = hi - lo;
  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    const int64_t j = lo + (int64_t)(hash_u32(seed ^ (uint32_t)(i * 2654435761u)) % (uint64_t)n);
    float g;
    if (vel && masking) {
      g = err[j] + (mu * vel[j] + grad[j] * scale);
    } else {
      g = grad[j] * scale + err[j];
      if (vel) g = mu * vel[j] + g;
    }
    smp[i] = fabsf(g);
  }
  __syncthreads();
  for (int k = 2; k <= S; k <<= 1) {
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < S; i += blockDim.x) {
        const int ix = i ^ jj;
        if (ix > i) {
          const float a = smp[i], b = smp[ix];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            smp[i] = b;
            smp[ix] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    int cut = (int)floorf((float)S * (1.f - keep_ratio));
    if (cut > S - 1) cut = S - 1;
    *thr_out = smp[cut];
  }
}

struct SelChunk {
  int64_t off;    // element offset (flat layout)
  int64_t len;
  int64_t list;   // slot offset of the owner's list for this bucket (in pairs)
  int64_t cnt;    // counter index of (bucket, owner)
};

// counts: this rank's per-(bucket, owner) counters (symmetric memory); idx/val: this rank's lists.
__global__ void __launch_bounds__(256) topk_select_kernel(const float* __restrict__ grad, float* __restrict__ err,
                                                          float* __restrict__ vel, const SelChunk* __restrict__ chunks,
                                                          int nchunks, float scale, float mu, int masking,
                                                          const float* __restrict__ thr_p, uint32_t* __restrict__ idx,
                                                          __half* __restrict__ val, int* __restrict__ counts) {
  const float thr = *thr_p;
  const int lane = threadIdx.x & 31;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const SelChunk ch = chunks[c];
    for (int64_t j0 = 0; j0 < ch.len; j0 += blockDim.x) {
      const int64_t j = j0 + threadIdx.x;
      bool keep = false;
      float g = 0.f;
      const int64_t i = ch.off + j;
      if (j < ch.len) {
        if (vel && masking) {
          const float u = mu * vel[i] + grad[i] * scale;
          g = err[i] + u;
          keep = fabsf(g) >= thr;
          vel[i] = keep ? 0.f : u;
        } else {
          g = grad[i] * scale + err[i];
          if (vel) {
            g = mu * vel[i] + g;
            vel[i] = g;
          }
          keep = fabsf(g) >= thr;
        }
        err[i] = keep ? 0.f : g;
      }
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      int base = 0;
      if (lane == 0 && m) base = atomicAdd(counts + ch.cnt, __popc(m));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (keep) {
        const int64_t slot = ch.list + base + __popc(m & ((1u << lane) - 1));
        idx[slot] = (uint32_t)i;
        val[slot] = __float2half(g);
      }
    }
  }
}

struct PeerList {
  int64_t idx;    // pointer to the peer's index array
  int64_t val;    // pointer to the peer's value array
  int64_t cnt;    // pointer to the peer's counters
};

// Owner side: red[idx] += val / N for every pair in every peer's list for (bucket, me).
__global__ void __launch_bounds__(256) topk_reduce_kernel(const PeerList* __restrict__ peers, int npeers,
                                                          const int64_t* const* flags, int slot, int64_t epoch,
                                                          int64_t list_off, int cnt_index, float* __restrict__ red,
                                                          float scale, uint64_t budget_ns, int* status) {
  if (!wait_peers(flags, npeers, slot, epoch, budget_ns, status)) return;
  for (int p = 0; p < npeers; ++p) {
    const uint32_t* ix = reinterpret_cast<const uint32_t*>(peers[p].idx) + list_off;
    const __half* vx = reinterpret_cast<const __half*>(peers[p].val) + list_off;
    const int n = reinterpret_cast<const volatile int*>(peers[p].cnt)[cnt_index];
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
      atomicAdd(red + __ldcg(ix + j), __half2float(__ldcg(vx + j)) * scale);
  }
}

int sm_count() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

// ------------------------------------------------------------------------------------- symmetric memory
// Allocates `bytes` of device memory (zeroed) and returns (pointer, 64-byte IPC handle).
std::tuple<int64_t, torch::Tensor> sym_alloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::dtype(torch::kUInt8));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), t};
}

int64_t sym_open(const torch::Tensor& handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void sym_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }
void sym_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

// Wraps raw device memory as a tensor view (no ownership).
torch::Tensor sym_view(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device) {
  const at::ScalarType st = dtype_code == 0 ? at::kFloat : dtype_code == 1 ? at::kBFloat16 : dtype_code == 2 ? at::kHalf
                                                                                                         : at::kLong;
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel},
                          torch::TensorOptions().dtype(st).device(torch::kCUDA, (c10::DeviceIndex)device));
}

// ------------------------------------------------------------------------------------- kernels
void comm_pack(const torch::Tensor& src, int64_t send_ptr, int64_t wire, int64_t lo, int64_t hi, double scale,
               torch::Tensor& bad) {
  c10::cuda::CUDAGuard g(src.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t n = hi - lo;
  if (n <= 0) return;
  const int grid = (int)std::min<int64_t>((n + 1023) / 1024, 2 * sm_count());
  void* send = reinterpret_cast<void*>(send_ptr);
  if (wire == W_F32)
    pack_kernel<W_F32><<<grid, 256, 0, st>>>(src.data_ptr<float>(), send, lo, hi, (float)scale, bad.data_ptr<int>());
  else if (wire == W_BF16)
    pack_kernel<W_BF16><<<grid, 256, 0, st>>>(src.data_ptr<float>(), send, lo, hi, (float)scale, bad.data_ptr<int>());
  else
    pack_kernel<W_F16><<<grid, 256, 0, st>>>(src.data_ptr<float>(), send, lo, hi, (float)scale, bad.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void comm_signal(int64_t flag_ptr, int64_t value) {
  signal_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<int64_t*>(flag_ptr), value);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// peers: int64 device tensor [N] of send-buffer pointers; flags: int64 device tensor [N] of flag-array pointers;
// chunks: int64 device tensor [nchunks, 2] (offset, length) in elements (offsets multiples of 8).
void comm_reduce(const torch::Tensor& peers, const torch::Tensor& flags, int64_t slot, int64_t epoch,
                 const torch::Tensor& chunks, torch::Tensor& out, int64_t wire, double scale, int64_t max_blocks,
                 double budget_s) {
  c10::cuda::CUDAGuard g(out.device());
  const int nch = (int)chunks.size(0);
  if (nch == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)std::min<int64_t>(nch, max_blocks > 0 ? max_blocks : sm_count());
  const uint64_t budget = (uint64_t)(budget_s * 1e9);
  int* status = status_ptr(out.device().index());
  auto P = reinterpret_cast<const void* const*>(peers.data_ptr<int64_t>());
  auto F = reinterpret_cast<const int64_t* const*>(flags.data_ptr<int64_t>());
  auto C = reinterpret_cast<const Chunk*>(chunks.data_ptr<int64_t>());
  const int np = (int)peers.numel();
  if (wire == W_F32)
    reduce_kernel<W_F32><<<grid, 256, 0, st>>>(P, F, np, (int)slot, epoch, C, nch, out.data_ptr<float>(), (float)scale, budget, status);
  else if (wire == W_BF16)
    reduce_kernel<W_BF16><<<grid, 256, 0, st>>>(P, F, np, (int)slot, epoch, C, nch, out.data_ptr<float>(), (float)scale, budget, status);
  else
    reduce_kernel<W_F16><<<grid, 256, 0, st>>>(P, F, np, (int)slot, epoch, C, nch, out.data_ptr<float>(), (float)scale, budget, status);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// segs: int64 device tensor [nsegs, 7] = (off, len, owner, cols, shadow_ld, shadow_ptr, start)
void comm_gather(const torch::Tensor& peers, const torch::Tensor& flags, int64_t slot, int64_t epoch,
                 const torch::Tensor& segs, torch::Tensor& local, int64_t max_blocks, double budget_s) {
  static_assert(sizeof(GatherSeg) == 7 * 8, "GatherSeg layout");
  c10::cuda::CUDAGuard g(local.device());
  const int ns = (int)segs.size(0);
  if (ns == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)std::min<int64_t>(ns, max_blocks > 0 ? max_blocks : sm_count());
  gather_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float* const*>(peers.data_ptr<int64_t>()),
                                      reinterpret_cast<const int64_t* const*>(flags.data_ptr<int64_t>()),
                                      (int)peers.numel(), (int)slot, epoch,
                                      reinterpret_cast<const GatherSeg*>(segs.data_ptr<int64_t>()), ns,
                                      local.data_ptr<float>(), (uint64_t)(budget_s * 1e9),
                                      status_ptr(local.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace br

namespace br {
// chunks: int64 [n, 2] (offset, length) of the parameters this rank owns; peers: int64 [N] param buffers
void comm_push(const torch::Tensor& params, const torch::Tensor& peers, int64_t me, const torch::Tensor& chunks,
               int64_t max_blocks) {
  c10::cuda::CUDAGuard g(params.device());
  const int n = (int)chunks.size(0);
  if (n == 0) return;
  const int grid = (int)std::min<int64_t>(n, max_blocks > 0 ? max_blocks : 2 * sm_count());
  push_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      params.data_ptr<float>(), reinterpret_cast<float* const*>(peers.data_ptr<int64_t>()), (int)peers.numel(),
      (int)me, reinterpret_cast<const Chunk*>(chunks.data_ptr<int64_t>()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// flag_peers: int64 [N] pointers to every rank's push-flag array (N int64 slots each)
void comm_signal_peers(const torch::Tensor& flag_peers, int64_t me, int64_t epoch) {
  c10::cuda::CUDAGuard g(flag_peers.device());
  signal_peers_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<int64_t* const*>(flag_peers.data_ptr<int64_t>()), (int)flag_peers.numel(), (int)me, epoch);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// chunks: int64 [n, 4] (off, len, owner, slot_off) of every parameter run of one bucket; recv_peers: int64 [N]
// receive-buffer pointers (this rank's own included)
void comm_pack_push(const torch::Tensor& grad, const torch::Tensor& recv_peers, int64_t me, int64_t slot_elems,
                    const torch::Tensor& chunks, int64_t wire, double scale, torch::Tensor& bad, int64_t max_blocks) {
  static_assert(sizeof(PushChunk) == 4 * 8, "PushChunk layout");
  c10::cuda::CUDAGuard g(grad.device());
  const int n = (int)chunks.size(0);
  if (n == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)std::min<int64_t>(n, max_blocks > 0 ? max_blocks : sm_count());
  auto R = reinterpret_cast<void* const*>(recv_peers.data_ptr<int64_t>());
  auto C = reinterpret_cast<const PushChunk*>(chunks.data_ptr<int64_t>());
  if (wire == W_F32)
    pack_push_kernel<W_F32><<<grid, 256, 0, st>>>(grad.data_ptr<float>(), R, (int)me, slot_elems, C, n, (float)scale,
                                                 bad.data_ptr<int>());
  else if (wire == W_BF16)
    pack_push_kernel<W_BF16><<<grid, 256, 0, st>>>(grad.data_ptr<float>(), R, (int)me, slot_elems, C, n, (float)scale,
                                                  bad.data_ptr<int>());
  else
    pack_push_kernel<W_F16><<<grid, 256, 0, st>>>(grad.data_ptr<float>(), R, (int)me, slot_elems, C, n, (float)scale,
                                                 bad.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void comm_signal_all(const torch::Tensor& flag_peers, int64_t me, int64_t slot, int64_t epoch, const torch::Tensor& bad) {
  c10::cuda::CUDAGuard g(flag_peers.device());
  signal_all_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<int64_t* const*>(flag_peers.data_ptr<int64_t>()), (int)flag_peers.numel(), (int)me, (int)slot,
      epoch, bad.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// chunks: int64 [n, 4] of the runs this rank owns in the bucket; recv_ptr/flags_ptr: this rank's buffers
void comm_reduce_local(int64_t recv_ptr, int64_t flags_ptr, int64_t npeers, int64_t slot, int64_t epoch,
                       int64_t slot_elems, const torch::Tensor& chunks, torch::Tensor& out, int64_t wire, double scale,
                       int64_t max_blocks, double budget_s) {
  c10::cuda::CUDAGuard g(out.device());
  const int n = (int)chunks.size(0);
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(n, max_blocks > 0 ? max_blocks : sm_count()));
  const void* R = reinterpret_cast<const void*>(recv_ptr);
  auto F = reinterpret_cast<const int64_t*>(flags_ptr);
  auto C = reinterpret_cast<const PushChunk*>(chunks.data_ptr<int64_t>());
  const uint64_t budget = (uint64_t)(budget_s * 1e9);
  int* status = status_ptr(out.device().index());
  if (wire == W_F32)
    reduce_local_kernel<W_F32><<<grid, 256, 0, st>>>(R, F, (int)npeers, (int)slot, epoch, slot_elems, C, n,
                                                    out.data_ptr<float>(), (float)scale, budget, status);
  else if (wire == W_BF16)
    reduce_local_kernel<W_BF16><<<grid, 256, 0, st>>>(R, F, (int)npeers, (int)slot, epoch, slot_elems, C, n,
                                                     out.data_ptr<float>(), (float)scale, budget, status);
  else
    reduce_local_kernel<W_F16><<<grid, 256, 0, st>>>(R, F, (int)npeers, (int)slot, epoch, slot_elems, C, n,
                                                    out.data_ptr<float>(), (float)scale, budget, status);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// skip (int32 [1]) = 1 if any rank flagged a non-finite gradient in the step (bit of `slot`'s flags), a wait
// timed out or the device status word is set; 0 otherwise
void comm_agree(int64_t flags_ptr, int64_t npeers, int64_t slot, int64_t epoch, torch::Tensor& skip, double budget_s) {
  c10::cuda::CUDAGuard g(skip.device());
  agree_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const int64_t*>(flags_ptr),
                                                              (int)npeers, (int)slot, epoch, skip.data_ptr<int>(),
                                                              (uint64_t)(budget_s * 1e9),
                                                              status_ptr(skip.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// waits for every other rank's push (this rank's flag slots >= epoch), then refreshes bf16 shadows
void comm_shadow_refresh(const torch::Tensor& params, int64_t push_flags_ptr, int64_t npeers, int64_t me,
                         int64_t epoch, const torch::Tensor& segs, int64_t max_blocks, double budget_s) {
  c10::cuda::CUDAGuard g(params.device());
  const int ns = (int)segs.size(0);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ns, max_blocks > 0 ? max_blocks : sm_count()));
  shadow_refresh_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      params.data_ptr<float>(), reinterpret_cast<const int64_t*>(push_flags_ptr), (int)npeers, (int)me, epoch,
      reinterpret_cast<const GatherSeg*>(segs.data_ptr<int64_t>()), ns, (uint64_t)(budget_s * 1e9),
      status_ptr(params.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace br

namespace br {
void topk_threshold(const torch::Tensor& grad, const torch::Tensor& err, c10::optional<torch::Tensor> vel, int64_t lo,
                    int64_t hi, double scale, double mu, int64_t sample, double keep_ratio, int64_t seed,
                    bool masking, torch::Tensor& thr_out) {
  int S = 1;
  while (S < std::min<int64_t>(sample, hi - lo)) S <<= 1;
  TORCH_CHECK(S <= 16384, "topk_threshold: sample size must be <= 16384");
  c10::cuda::CUDAGuard g(grad.device());
  const size_t sm = (size_t)S * sizeof(float);
  if (sm > 48 * 1024)
    C10_CUDA_CHECK(cudaFuncSetAttribute(topk_threshold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  topk_threshold_kernel<<<1, 1024, sm, at::cuda::getCurrentCUDAStream()>>>(
      grad.data_ptr<float>(), err.data_ptr<float>(), vel.has_value() ? vel->data_ptr<float>() : nullptr, lo, hi,
      (float)scale, (float)mu, S, (float)keep_ratio, (uint32_t)seed, masking ? 1 : 0, thr_out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// chunks: int64 [n, 4] = (off, len, list_slot, counter_index)
void topk_select(const torch::Tensor& grad, torch::Tensor& err, c10::optional<torch::Tensor> vel,
                 const torch::Tensor& chunks, double scale, double mu, bool masking, const torch::Tensor& thr,
                 int64_t idx_ptr, int64_t val_ptr, int64_t cnt_ptr) {
  static_assert(sizeof(SelChunk) == 32, "SelChunk layout");
  c10::cuda::CUDAGuard g(grad.device());
  const int n = (int)chunks.size(0);
  if (n == 0) return;
  topk_select_kernel<<<std::min(n, 4 * sm_count()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      grad.data_ptr<float>(), err.data_ptr<float>(), vel.has_value() ? vel->data_ptr<float>() : nullptr,
      reinterpret_cast<const SelChunk*>(chunks.data_ptr<int64_t>()), n, (float)scale, (float)mu, masking ? 1 : 0,
      thr.data_ptr<float>(),
      reinterpret_cast<uint32_t*>(idx_ptr), reinterpret_cast<__half*>(val_ptr), reinterpret_cast<int*>(cnt_ptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// peers: int64 [N, 3] = (idx ptr, val ptr, counters ptr) of every rank
void topk_reduce(const torch::Tensor& peers, const torch::Tensor& flags, int64_t slot, int64_t epoch, int64_t list_off,
                 int64_t cnt_index, torch::Tensor& red, double scale, int64_t max_blocks, double budget_s) {
  static_assert(sizeof(PeerList) == 24, "PeerList layout");
  c10::cuda::CUDAGuard g(red.device());
  topk_reduce_kernel<<<(int)std::max<int64_t>(1, max_blocks), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const PeerList*>(peers.data_ptr<int64_t>()), (int)peers.size(0),
      reinterpret_cast<const int64_t* const*>(flags.data_ptr<int64_t>()), (int)slot, epoch, list_off, (int)cnt_index,
      red.data_ptr<float>(), (float)scale, (uint64_t)(budget_s * 1e9), status_ptr(red.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace br
