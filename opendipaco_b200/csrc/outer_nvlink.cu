// Cross-GPU DiLoCo outer step over NVLink peer memory (one process per GPU).
//
// Every rank holds the whole bank's address space in symmetric buffers (same offsets
// on all ranks): DELTA (each rank's weighted pseudo-gradient partial, written by the
// local ACC pass) and GLOB (the authoritative global weights). For every shared
// module key, the ranks whose paths use it (its sharers) split its elements into
// contiguous slices; rank i owns slice i.
//
// outer_nvlink_apply (one launch per round):
//   1. CTA 0 publishes "my DELTA is complete" to every peer's signal pad (the ACC
//      kernel finished before this launch on the same stream); every CTA then waits,
//      bounded, until all ranks have published this round's epoch.
//   2. For each element of each slice it owns: acc = sum over sharers s, in rank
//      order, of DELTA_s[e] (peer loads over NVLink, L2-only); d = acc * inv_den *
//      scale; Nesterov with this rank's momentum shard; new global written with peer
//      stores into GLOB_s[e] of every sharer s (this rank included).
// outer_nvlink_bcast (next launch):
//   3. CTA 0 publishes "my peer stores are complete"; every CTA waits for all ranks;
//      then the fresh globals are copied into this GPU's working copies (fp32 + bf16).
//
// So per round each rank reads (g-1)/g and writes (g-1)/g of every module it shares
// over NVLink (two-shot reduce-scatter + all-gather), fused with the reduction, the
// optimizer and the write-back.
//
// Compressed mode (int4): before APPLY, outer_nvlink_quant turns each rank's DELTA
// partial (plus its error-feedback residual) into 4-bit codes with one absmax/7 scale per
// 128 elements (symmetric buffers QD, QS) and keeps what the codes miss as the residual
// for the next round. APPLY then reads the sharers' codes and scales instead of their
// fp32 partials (0.53 instead of 4 bytes per element over NVLink) and dequantises them in
// registers inside the same reduction. Waits never spin forever: after kWaitBoundNs they
// record ERR_TIMEOUT_PEER and the kernel returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

constexpr int kMaxSharers = 8;

struct NvKey {
  long long off;    // element offset of the key in the symmetric DELTA / GLOB buffers
  long long s0, s1; // this rank's slice [s0, s1) (multiples of 4)
  long long chunk0; // first chunk of this slice in the flat chunk space
  int nsh;          // number of sharer ranks
  int sh[kMaxSharers];
  float scale, inv_den;
  int quant;        // 1: read the sharers' int4 codes + scales instead of their fp32 partials
};

constexpr int kNvChunk = 4096;

ODP_DEVICE void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
ODP_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
ODP_DEVICE float4 ld_cg4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Publish `epoch` on channel `ch` of every rank's pad, then wait for all ranks.
// pads[r] points at rank r's pad: uint32 [2][world]. Returns false on timeout.
ODP_DEVICE bool cross_gpu_barrier(const unsigned long long* pads, int rank, int world, int ch, unsigned epoch,
                                  int* err, bool publish) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (publish) {
      __threadfence_system();
      for (int r = 0; r < world; ++r) {
        unsigned* pad = reinterpret_cast<unsigned*>(pads[r]);
        st_release_sys(pad + ch * world + rank, epoch);
      }
    }
    const unsigned* mine = reinterpret_cast<const unsigned*>(pads[rank]) + ch * world;
    ok = 1;
    unsigned long long t0 = globaltimer();
    for (int r = 0; r < world; ++r) {
      while (ld_acquire_sys(mine + r) < epoch) {
        if (globaltimer() - t0 > kWaitBoundNs) {
          record_error(err, ERR_TIMEOUT_PEER);
          ok = 0;
          break;
        }
      }
      if (!ok) break;
    }
  }
  __syncthreads();
  return ok != 0;
}

constexpr int kQGroup = 128;

// Quantise this rank's partials: one warp per 128-element group of the regions listed in
// `regs` (off, n, group0), x = delta + res, codes q in [-7, 7] stored as q + 8 (two per
// byte, element e in the low nibble of byte e/2 when e is even), res = x - q * scale.
struct NvRegion {
  long long off, n, group0;
};

__global__ void outer_nvlink_quant_kernel(const NvRegion* __restrict__ regs, int nregs, long long total_groups,
                                          const float* __restrict__ delta, float* __restrict__ res,
                                          uint8_t* __restrict__ qd, float* __restrict__ qs) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= total_groups) return;
  int lo = 0, hi = nregs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (regs[mid].group0 <= w) lo = mid;
    else hi = mid - 1;
  }
  const NvRegion r = regs[lo];
  const long long e = r.off + (w - r.group0) * kQGroup + lane * 4;
  const float4 dv = *reinterpret_cast<const float4*>(delta + e);
  const float4 rv = *reinterpret_cast<const float4*>(res + e);
  float x[4] = {__fadd_rn(dv.x, rv.x), __fadd_rn(dv.y, rv.y), __fadd_rn(dv.z, rv.z), __fadd_rn(dv.w, rv.w)};
  float am = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  am = warp_max(am);
  const float sc = am / 7.f;
  const float safe = sc > 0.f ? sc : 1.f;
  uint32_t codes = 0;
  float r4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = (int)fminf(fmaxf(rintf(x[i] / safe), -7.f), 7.f);
    r4[i] = __fsub_rn(x[i], __fmul_rn((float)q, sc));
    codes |= (uint32_t)(q + 8) << (4 * i);
  }
  *reinterpret_cast<float4*>(res + e) = make_float4(r4[0], r4[1], r4[2], r4[3]);
  *reinterpret_cast<uint16_t*>(qd + e / 2) = (uint16_t)codes;
  if (lane == 0) qs[(r.off + (w - r.group0) * kQGroup) / kQGroup] = sc;
}

__global__ void outer_nvlink_apply_kernel(const NvKey* __restrict__ keys, int nkeys, long long total_chunks,
                                          const unsigned long long* __restrict__ delta_ptrs,
                                          const unsigned long long* __restrict__ glob_ptrs,
                                          const unsigned long long* __restrict__ pads, float* __restrict__ mom,
                                          int rank, int world, unsigned epoch, float lr, float m, int nesterov,
                                          int first, float* __restrict__ sq_part, int* err,
                                          const unsigned long long* __restrict__ qd_ptrs,
                                          const unsigned long long* __restrict__ qs_ptrs) {
  if (!cross_gpu_barrier(pads, rank, world, 0, epoch, err, blockIdx.x == 0)) return;
  __shared__ float red[8];
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    int lo = 0, hi = nkeys - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (keys[mid].chunk0 <= ch) lo = mid;
      else hi = mid - 1;
    }
    const NvKey k = keys[lo];
    const long long e0 = k.s0 + (ch - k.chunk0) * kNvChunk;
    const long long e1 = min(e0 + kNvChunk, k.s1);
    float sq = 0.f;
    const float* gl = reinterpret_cast<const float*>(glob_ptrs[rank]) + k.off;
    for (long long e = e0 + threadIdx.x * 4; e < e1; e += blockDim.x * 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < k.nsh; ++j) {
        float4 d;
        if (k.quant) {  // int4 codes + group scale of sharer j, dequantised in registers
          const long long ge = k.off + e;
          const uint16_t c = *reinterpret_cast<const volatile uint16_t*>(
              reinterpret_cast<const uint8_t*>(qd_ptrs[k.sh[j]]) + ge / 2);
          const float sc = *reinterpret_cast<const volatile float*>(
              reinterpret_cast<const float*>(qs_ptrs[k.sh[j]]) + ge / kQGroup);
          d = make_float4(__fmul_rn((float)((int)(c & 15u) - 8), sc), __fmul_rn((float)((int)((c >> 4) & 15u) - 8), sc),
                          __fmul_rn((float)((int)((c >> 8) & 15u) - 8), sc),
                          __fmul_rn((float)((int)((c >> 12) & 15u) - 8), sc));
        } else {
          d = ld_cg4(reinterpret_cast<const float*>(delta_ptrs[k.sh[j]]) + k.off + e);
        }
        acc.x = __fadd_rn(acc.x, d.x);
        acc.y = __fadd_rn(acc.y, d.y);
        acc.z = __fadd_rn(acc.z, d.z);
        acc.w = __fadd_rn(acc.w, d.w);
      }
      const float4 gv = *reinterpret_cast<const float4*>(gl + e);
      float4 mb = *reinterpret_cast<const float4*>(mom + k.off + e);
      float a4[4] = {acc.x, acc.y, acc.z, acc.w}, g4[4] = {gv.x, gv.y, gv.z, gv.w};
      float b4[4] = {mb.x, mb.y, mb.z, mb.w}, n4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float d = __fmul_rn(__fmul_rn(a4[i], k.inv_den), k.scale);
        sq += d * d;
        const float b = first ? d : __fadd_rn(__fmul_rn(b4[i], m), d);
        b4[i] = b;
        const float upd = nesterov ? __fadd_rn(d, __fmul_rn(m, b)) : b;
        n4[i] = __fadd_rn(g4[i], __fmul_rn(-lr, upd));
      }
      *reinterpret_cast<float4*>(mom + k.off + e) = make_float4(b4[0], b4[1], b4[2], b4[3]);
      const float4 nv = make_float4(n4[0], n4[1], n4[2], n4[3]);
      for (int j = 0; j < k.nsh; ++j)
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(glob_ptrs[k.sh[j]]) + k.off + e) = nv;
    }
    if (sq_part) {
      sq = warp_sum(sq);
      if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sq;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)blockDim.x / 32; ++w) t += red[w];
        sq_part[ch] = t;
      }
      __syncthreads();
    }
  }
}

// Copy the fresh globals into this GPU's working copies after all ranks' stores.
struct NvCopy {
  const float* src;
  float* dst32;
  __nv_bfloat16* dst16;
  long long n;
  long long chunk0;
};

__global__ void outer_nvlink_bcast_kernel(const NvCopy* __restrict__ cps, int ncp, long long total_chunks,
                                          const unsigned long long* __restrict__ pads, int rank, int world,
                                          unsigned epoch, int* err) {
  if (!cross_gpu_barrier(pads, rank, world, 1, epoch, err, blockIdx.x == 0)) return;
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    int lo = 0, hi = ncp - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (cps[mid].chunk0 <= ch) lo = mid;
      else hi = mid - 1;
    }
    const NvCopy c = cps[lo];
    const long long e0 = (ch - c.chunk0) * kNvChunk;
    const long long e1 = min(e0 + kNvChunk, c.n);
    for (long long e = e0 + threadIdx.x * 4; e < e1; e += blockDim.x * 4) {
      const float4 v = ld_cg4(c.src + e);
      *reinterpret_cast<float4*>(c.dst32 + e) = v;
      *reinterpret_cast<uint2*>(c.dst16 + e) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
    }
  }
}

}  // namespace odp

void outer_nvlink_apply(torch::Tensor keys, int64_t nkeys, int64_t total_chunks, torch::Tensor delta_ptrs,
                        torch::Tensor glob_ptrs, torch::Tensor pads, torch::Tensor mom, int64_t rank, int64_t world,
                        int64_t epoch, double lr, double m, bool nesterov, bool first, torch::Tensor sq_part,
                        torch::Tensor err, c10::optional<torch::Tensor> qd_ptrs, c10::optional<torch::Tensor> qs_ptrs) {
  static_assert(sizeof(odp::NvKey) == 80, "NvKey layout");
  c10::cuda::CUDAGuard guard(mom.device());
  TORCH_CHECK(world <= 64, "outer_nvlink: world too large");
  // Always launch (even with no owned slices): every rank must take part in the barrier.
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total_chunks, 148 * 4));
  odp::outer_nvlink_apply_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::NvKey*>(keys.data_ptr()), (int)nkeys, total_chunks,
      reinterpret_cast<const unsigned long long*>(delta_ptrs.data_ptr()),
      reinterpret_cast<const unsigned long long*>(glob_ptrs.data_ptr()),
      reinterpret_cast<const unsigned long long*>(pads.data_ptr()), mom.data_ptr<float>(), (int)rank, (int)world,
      (unsigned)epoch, (float)lr, (float)m, nesterov ? 1 : 0, first ? 1 : 0, sq_part.data_ptr<float>(),
      err.data_ptr<int>(),
      qd_ptrs.has_value() ? reinterpret_cast<const unsigned long long*>(qd_ptrs->data_ptr()) : nullptr,
      qs_ptrs.has_value() ? reinterpret_cast<const unsigned long long*>(qs_ptrs->data_ptr()) : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// regs: int64 [nregs][3] = (element offset, elements, first group); offsets and sizes are
// multiples of 128.
void outer_nvlink_quant(torch::Tensor regs, int64_t nregs, int64_t total_groups, torch::Tensor delta,
                        torch::Tensor res, torch::Tensor qd, torch::Tensor qs) {
  static_assert(sizeof(odp::NvRegion) == 24, "NvRegion layout");
  c10::cuda::CUDAGuard guard(delta.device());
  if (total_groups == 0) return;
  odp::outer_nvlink_quant_kernel<<<(unsigned)((total_groups * 32 + 255) / 256), 256, 0,
                                   at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::NvRegion*>(regs.data_ptr()), (int)nregs, total_groups, delta.data_ptr<float>(),
      res.data_ptr<float>(), qd.data_ptr<uint8_t>(), qs.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void outer_nvlink_bcast(torch::Tensor cps, int64_t ncp, int64_t total_chunks, torch::Tensor pads, int64_t rank,
                        int64_t world, int64_t epoch, torch::Tensor err) {
  static_assert(sizeof(odp::NvCopy) == 40, "NvCopy layout");
  c10::cuda::CUDAGuard guard(pads.device());
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total_chunks, 148 * 4));
  odp::outer_nvlink_bcast_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::NvCopy*>(cps.data_ptr()), (int)ncp, total_chunks,
      reinterpret_cast<const unsigned long long*>(pads.data_ptr()), (int)rank, (int)world, (unsigned)epoch,
      err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t outer_nvlink_chunk_elems() { return odp::kNvChunk; }
