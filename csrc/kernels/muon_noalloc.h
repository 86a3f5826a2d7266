// Allocation-free C entry point for the Muon momentum + normalisation step.
//
// This entry point has no counterpart in the reference project (a TypeScript trainer); it exists for
// callers of this library that cannot allocate device memory themselves: runtimes that plan all
// device memory ahead of time and hand kernels only the buffers they planned, and host code that
// must not call cudaMalloc/cudaFree because those calls can synchronise the device. Such callers
// pass their inputs and outputs; the scratch the kernel needs lives in a fixed-size array compiled
// into this library.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest number of matrices one call accepts (the scratch holds one float per matrix).
#define BR_MUON_NOALLOC_MAX_MATRICES 4096

// For S matrices of n elements each, stored back to back (matrix s at offset s*n):
//   mom[s] = mu * mom[s] + (1 - mu) * grad[s]                 (updated in place)
//   g'     = (1 - mu) * grad[s] + mu * mom[s]                  (Nesterov)
//   x_out[s] = bf16(g' / (||g'||_F * 1.02 + 1e-6))
// which is the same result as the library's list-based `muon_prepare`.
// All pointers are device pointers; work is queued on `stream` and the call returns without waiting.
// Returns cudaSuccess, cudaErrorInvalidValue (S outside [1, BR_MUON_NOALLOC_MAX_MATRICES], n < 1 or a
// null pointer), or the error of the set-up or launch.
//
// Scratch: a file-scope __device__ array that every GPU loading the library holds until exit. The first
// call on each device looks up its address (cudaGetSymbolAddress) with that device current and keeps it
// for the life of the process; make that first call before any stream capture. A caller that resets a
// device (cudaDeviceReset) must not use this entry point on that device again in the same process: the
// kept address belongs to the destroyed context. Every call shares the array and clears the part it uses, so
// calls whose kernels overlap on the GPU (different streams, or different host threads, on one device)
// race and must be ordered by the caller.
cudaError_t br_muon_normalize_noalloc(const float* grad, float* mom, __nv_bfloat16* x_out, int S, int64_t n, float mu,
                                      cudaStream_t stream);

#ifdef __cplusplus
}
#endif
