// Allocation-free variant of the per-path gradient-norm clip coefficient. The interface,
// its limits and the callers it serves are described in clip_noalloc.h. This file has no
// counterpart in the reference.
//
// Two launches on the caller's stream, the same math and reduction order as
// grad_clip_coef (adam.cu):
//   1. grid (nblk, G) x 256 threads: block b of path g sums the squares of elements
//      [b * 65536, min((b + 1) * 65536, P)) with float4 loads and writes one partial to
//      scratch[g * nblk + b];
//   2. G blocks x 256 threads: path g adds its nblk partials in a fixed tree order and
//      writes norm and coef.
// The scratch lives in the static device array below instead of a caller-provided buffer.
#include "clip_noalloc.h"

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace {

constexpr int kBlock = 256;
constexpr long long kElemsPerBlock = 1LL << 16;
constexpr size_t kScratchFloats = (size_t)ODP_NOALLOC_MAX_GROUPS * ODP_NOALLOC_MAX_BLOCKS;  // 1 MiB
constexpr int kMaxDevices = 64;

}  // namespace

// The scratch: one 1 MiB array per device, shared by every call on that device. Host code
// must not hand this name to a kernel (on the host it is only a stand-in for the symbol);
// it passes the device address that cudaGetSymbolAddress returns.
static __device__ __align__(256) float odp_clip_noalloc_scratch[kScratchFloats];

namespace {

float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_setup_mu;

__global__ void noalloc_sumsq_kernel(const float* __restrict__ g, long long P, long long stride, int nblk,
                                     float* __restrict__ part) {
  const int grp = blockIdx.y, b = blockIdx.x;
  const float* base = g + grp * stride;
  const long long e0 = (long long)b * kElemsPerBlock;
  const long long e1 = min(e0 + kElemsPerBlock, P);
  float s = 0.f;
  for (long long i = e0 + threadIdx.x * 4; i < e1; i += kBlock * 4) {
    if (i + 4 <= e1) {
      const float4 v = *reinterpret_cast<const float4*>(base + i);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    } else {
      for (long long j = i; j < e1; ++j) s += base[j] * base[j];
    }
  }
  __shared__ float red[kBlock / 32];
  s = odp::warp_sum(s);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kBlock / 32; ++w) t += red[w];
    part[(long long)grp * nblk + b] = t;
  }
}

__global__ void noalloc_coef_kernel(const float* __restrict__ part, int nblk, float max_norm,
                                    float* __restrict__ coef, float* __restrict__ norm_out) {
  const int grp = blockIdx.x;
  __shared__ float red[kBlock];
  float s = 0.f;
  for (int i = threadIdx.x; i < nblk; i += kBlock) s += part[(long long)grp * nblk + i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = kBlock / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float n = sqrtf(red[0]);
    if (norm_out) norm_out[grp] = n;
    coef[grp] = max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
  }
}

int reject(int code, const char* why) {
  fprintf(stderr, "odp_grad_clip_coef_noalloc: %s\n", why);
  return code;
}

// True when `p` is device (or managed) memory of device `dev`. Called only once the entry
// point has checked that no earlier error was pending, so an error left behind here was
// recorded by this query and is the one to clear.
bool on_device(const void* p, int dev) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == dev;
}

// Device address of the scratch array on the current device; looked up once per device.
int scratch_address(int dev, float** out) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, odp_clip_noalloc_scratch);
    if (e != cudaSuccess) {
      fprintf(stderr, "odp_grad_clip_coef_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
              cudaGetErrorString(e));
      return (int)e;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace

extern "C" int odp_grad_clip_coef_noalloc(const float* grads, long long P, long long stride, int G, float max_norm,
                                          float* coef, float* norm_out, cudaStream_t stream) {
  if (grads == nullptr || coef == nullptr || P <= 0 || G <= 0 || stride < P)
    return reject(ODP_NOALLOC_EARG, "need grads and coef, P > 0, G > 0 and stride >= P");
  if (G > ODP_NOALLOC_MAX_GROUPS)
    return reject(ODP_NOALLOC_ETOO_MANY_GROUPS, "G is above ODP_NOALLOC_MAX_GROUPS (64 paths per call)");
  const long long nblk = (P + kElemsPerBlock - 1) / kElemsPerBlock;
  if (nblk > ODP_NOALLOC_MAX_BLOCKS)
    return reject(ODP_NOALLOC_ETOO_LONG, "P is above 4096 * 65536 elements per path");
  if ((reinterpret_cast<uintptr_t>(grads) & 15u) != 0 || (stride & 3) != 0)
    return reject(ODP_NOALLOC_EALIGN, "grads must be 16-byte aligned and stride a multiple of 4");
  // An error an earlier call left pending is returned as it is (and left pending): the
  // caller sees its own failure, and the launch checks below report only these launches.
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return (int)e;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return reject(ODP_NOALLOC_EDEVICE, "device ordinal above 63");
  int stream_dev = dev;
  e = cudaStreamGetDevice(stream, &stream_dev);
  if (e != cudaSuccess) return (int)e;
  if (stream_dev != dev) return reject(ODP_NOALLOC_EDEVICE, "the stream belongs to another device than the current one");
  if (!on_device(grads, dev) || !on_device(coef, dev) || (norm_out != nullptr && !on_device(norm_out, dev)))
    return reject(ODP_NOALLOC_EDEVICE, "grads, coef and norm_out must be memory of the current device");
  float* scratch = nullptr;
  const int rc = scratch_address(dev, &scratch);
  if (rc != 0) return rc;
  noalloc_sumsq_kernel<<<dim3((unsigned)nblk, (unsigned)G), kBlock, 0, stream>>>(grads, P, stride, (int)nblk,
                                                                                 scratch);
  e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  noalloc_coef_kernel<<<(unsigned)G, kBlock, 0, stream>>>(scratch, (int)nblk, max_norm, coef, norm_out);
  return (int)cudaGetLastError();
}
