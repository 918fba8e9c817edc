// Allocation-free entry point for the per-path gradient-norm clip coefficient.
//
// This entry point has no counterpart in the reference: it exists only in this library.
// It is for callers that cannot allocate GPU memory: a serving or training process that
// reserved all device memory up front for its own pool (a cudaMalloc would fail or
// break its accounting), a real-time step loop where an allocation's latency or its
// implicit synchronization is not allowed, and plain C code that links this library
// without torch and so has no caching allocator to draw scratch from. The usual path
// (`grad_clip_coef` in adam.cu, wrapped by `ops.adam.clip_coef`) needs a caller-
// provided scratch tensor of G * ceil(P / 65536) floats; this one keeps that scratch in
// a fixed static device array instead, so the caller supplies only inputs and outputs.
//
// What it computes, for every path g < G of a [G][stride] fp32 gradient buffer:
//   norm[g] = sqrt(sum_{i < P} grads[g * stride + i]^2)
//   coef[g] = max_norm > 0 ? min(1, max_norm / (norm[g] + 1e-6)) : 1
// with the same fixed-order reduction as grad_clip_coef, so the two give the same results.
//
// Limits (the size of the static scratch array, 1 MiB, held by every GPU that loads
// the library until the process exits):
//   G <= ODP_NOALLOC_MAX_GROUPS, and ceil(P / 65536) <= ODP_NOALLOC_MAX_BLOCKS
//   (P <= 268,435,456 elements per path). Larger sizes are rejected, nothing launched.
// Requirements: `grads` 16-byte aligned, `stride` a multiple of 4 and >= P; all pointers
// on the current device; `norm_out` may be NULL.
//
// Set-up: the first call on each device looks up the device address of the scratch
// array (cudaGetSymbolAddress) with that device current. Make that first call before
// any stream capture begins on that device. The address is cached for the life of the
// process: it assumes the device's primary context lives that long. After a
// cudaDeviceReset (or any teardown of the primary context) the cached address is stale
// and the entry point must not be called again in that process.
//
// Errors: an error already pending on the calling thread (cudaPeekAtLastError) is
// returned unchanged before anything is done, and stays pending. `stream` must belong to
// the current device (cudaStreamGetDevice), else ODP_NOALLOC_EDEVICE.
//
// Sharing: every call on a device uses the same scratch array, and the array keeps what
// the last call left in it. Each call overwrites every scratch slot it later reads, so
// nothing needs to start at zero. Calls whose kernels overlap on the GPU (different
// streams without ordering between them, or different host threads) race on the array
// and can return each other's sums: order them on one stream or serialize them.
//
// Returns 0 on success; a negative ODP_NOALLOC_E* code when the arguments are rejected
// (a one-line reason is also printed to stderr); otherwise the cudaError_t of the failed
// CUDA call. It never calls cudaMalloc, cudaFree or any allocating library routine.
#pragma once

#include <cuda_runtime.h>

#define ODP_NOALLOC_MAX_GROUPS 64
#define ODP_NOALLOC_MAX_BLOCKS 4096

#define ODP_NOALLOC_ETOO_MANY_GROUPS (-1)
#define ODP_NOALLOC_ETOO_LONG (-2)
#define ODP_NOALLOC_EALIGN (-3)
#define ODP_NOALLOC_EARG (-4)
#define ODP_NOALLOC_EDEVICE (-5)

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int odp_grad_clip_coef_noalloc(const float* grads, long long P,
                                                                       long long stride, int G, float max_norm,
                                                                       float* coef, float* norm_out,
                                                                       cudaStream_t stream);

#ifdef __cplusplus
}
#endif
