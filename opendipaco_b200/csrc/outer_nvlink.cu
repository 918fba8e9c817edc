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
//      then the fresh globals are copied into this GPU's working copies (fp32 + bf16),
//      each global read once for all of its local sharers.
// Guard: an element whose pseudo-gradient is not finite is not applied (global and
// momentum unchanged) and is counted in a status word the host reads after the round.
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
// registers inside the same reduction.
//
// Sparse mode (top-k): outer_nvlink_topk keeps, in every 4096-element block of each
// rank's partial (plus residual), the k = ceil(density * len) entries of largest
// magnitude (exact radix select, ties in index order) as (uint16 index, fp32 value)
// pairs in symmetric buffers; the dropped entries stay in the residual. APPLY then adds
// the sharers' pairs of its block into a zeroed shared-memory block, sharer by sharer
// (deterministic), and runs the same update. Key regions and slices are 4096-aligned in
// this mode, so an APPLY chunk is exactly one block. Waits never spin forever: after the
// bound passed at launch (peer_wait_bound_ns, 2 s by default) they record ERR_TIMEOUT_PEER
// and the kernel returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "outer_common.cuh"

namespace odp {

constexpr int kMaxSharers = 8;

struct NvKey {
  long long off;    // element offset of the key in the symmetric DELTA / GLOB buffers
  long long s0, s1; // this rank's slice [s0, s1) (multiples of 4)
  long long chunk0; // first chunk of this slice in the flat chunk space
  int nsh;          // number of sharer ranks
  int sh[kMaxSharers];
  float scale, inv_den;
  int quant;        // 1: the sharers' int4 codes + scales; 2: their top-k (index, value) pairs
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
                                  int* err, bool publish, unsigned long long bound_ns) {
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
        if (globaltimer() - t0 > bound_ns) {
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

// Block-wide exclusive prefix sum of one value per thread (256 threads); returns the
// exclusive prefix, writes the total.
ODP_DEVICE unsigned block_excl_scan256(unsigned v, unsigned* total) {
  __shared__ unsigned wsum[8];
  const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
  unsigned x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  unsigned before = 0, all = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    before += i < w ? wsum[i] : 0u;
    all += wsum[i];
  }
  __syncthreads();
  *total = all;
  return before + x - v;
}

constexpr int kSpPer = kNvChunk / 256;  // elements per thread in the top-k kernel
constexpr uint16_t kSpEmpty = 0xFFFF;

// One 256-thread CTA per 4096-element block of the regions in `regs` (off, n = the key's
// true size, group0 = the region's first block in launch order). Keys: |x| bits + 1 for
// valid elements (0 for the block's tail past n), so the k-th largest key is found by a
// 4-pass 8-bit radix select. Output slots are indexed by the block's position in the
// arena ((off + b * 4096) / 4096) and padded with kSpEmpty.
__global__ void __launch_bounds__(256) outer_nvlink_topk_kernel(const NvRegion* __restrict__ regs, int nregs,
                                                                double density, int kcap,
                                                                const float* __restrict__ delta,
                                                                float* __restrict__ res, uint16_t* __restrict__ spi,
                                                                float* __restrict__ spv) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_digit, s_remain;
  const long long blk = blockIdx.x;
  int lo = 0, hi = nregs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (regs[mid].group0 <= blk) lo = mid;
    else hi = mid - 1;
  }
  const NvRegion r = regs[lo];
  const long long b = blk - r.group0;
  const long long start = r.off + b * kNvChunk;
  const int len = (int)min((long long)kNvChunk, r.n - b * kNvChunk);
  const int kb = min(kcap, max(1, (int)ceil(density * (double)len)));
  const int t = threadIdx.x, i0 = t * kSpPer;
  float x[kSpPer];
  unsigned key[kSpPer];
#pragma unroll
  for (int v = 0; v < kSpPer / 4; ++v) {
    const float4 dv = *reinterpret_cast<const float4*>(delta + start + i0 + 4 * v);
    const float4 rv = *reinterpret_cast<const float4*>(res + start + i0 + 4 * v);
    x[4 * v] = __fadd_rn(dv.x, rv.x);
    x[4 * v + 1] = __fadd_rn(dv.y, rv.y);
    x[4 * v + 2] = __fadd_rn(dv.z, rv.z);
    x[4 * v + 3] = __fadd_rn(dv.w, rv.w);
  }
#pragma unroll
  for (int c = 0; c < kSpPer; ++c) key[c] = i0 + c < len ? __float_as_uint(fabsf(x[c])) + 1u : 0u;
  // radix select: prefix of the kb-th largest key, 8 bits a pass from the top
  unsigned prefix = 0, mask = 0, remain = (unsigned)kb;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[t] = 0;
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kSpPer; ++c)
      if ((key[c] & mask) == prefix) atomicAdd(&hist[(key[c] >> shift) & 255u], 1u);
    __syncthreads();
    if (t < 32) {
      // lane l sums bins [255 - 8l - 7, 255 - 8l] (highest bins first)
      unsigned cnt = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) cnt += hist[255 - 8 * t - j];
      unsigned cum = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, cum, o);
        if (t >= o) cum += y;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, cum >= remain);
      const int L = hit ? __ffs(hit) - 1 : -1;  // remain <= count of candidates, so some lane hits
      if (L < 0 && t == 0) {
        s_digit = 0;
        s_remain = remain;
      }
      if (t == L) {
        unsigned before = cum - cnt;
        for (int j = 0; j < 8; ++j) {
          const int bin = 255 - 8 * t - j;
          if (before + hist[bin] >= remain) {
            s_digit = (unsigned)bin;
            s_remain = remain - before;
            break;
          }
          before += hist[bin];
        }
      }
    }
    __syncthreads();
    prefix |= s_digit << shift;
    mask |= 0xFFu << shift;
    remain = s_remain;
    __syncthreads();
  }
  // keep key > T, and the first `remain` keys == T in index order
  unsigned n_eq = 0;
#pragma unroll
  for (int c = 0; c < kSpPer; ++c) n_eq += key[c] == prefix;
  unsigned tot;
  unsigned eq_before = block_excl_scan256(n_eq, &tot);
  bool keep[kSpPer];
  unsigned n_keep = 0;
#pragma unroll
  for (int c = 0; c < kSpPer; ++c) {
    bool k = key[c] > prefix;
    if (key[c] == prefix) {
      k = eq_before < remain;
      ++eq_before;
    }
    keep[c] = k;
    n_keep += k;
  }
  unsigned pos = block_excl_scan256(n_keep, &tot);
  uint16_t* oi = spi + (start / kNvChunk) * kcap;
  float* ov = spv + (start / kNvChunk) * kcap;
  float rnew[kSpPer];
#pragma unroll
  for (int c = 0; c < kSpPer; ++c) {
    rnew[c] = keep[c] ? 0.f : (i0 + c < len ? x[c] : 0.f);
    if (keep[c]) {
      oi[pos] = (uint16_t)(i0 + c);
      ov[pos] = x[c];
      ++pos;
    }
  }
  for (int i = (int)tot + t; i < kcap; i += 256) {
    oi[i] = kSpEmpty;
    ov[i] = 0.f;
  }
#pragma unroll
  for (int v = 0; v < kSpPer / 4; ++v)
    *reinterpret_cast<float4*>(res + start + i0 + 4 * v) =
        make_float4(rnew[4 * v], rnew[4 * v + 1], rnew[4 * v + 2], rnew[4 * v + 3]);
}

__global__ void outer_nvlink_apply_kernel(const NvKey* __restrict__ keys, int nkeys, long long total_chunks,
                                          const unsigned long long* __restrict__ delta_ptrs,
                                          const unsigned long long* __restrict__ glob_ptrs,
                                          const unsigned long long* __restrict__ pads, float* __restrict__ mom,
                                          int rank, int world, unsigned epoch, float lr, float m, int nesterov,
                                          int first, float* __restrict__ sq_part, int* err,
                                          const unsigned long long* __restrict__ qd_ptrs,
                                          const unsigned long long* __restrict__ qs_ptrs, int kcap,
                                          unsigned long long wait_ns, int* status) {
  if (!cross_gpu_barrier(pads, rank, world, 0, epoch, err, blockIdx.x == 0, wait_ns)) return;
  __shared__ __align__(16) float dense[kNvChunk];  // top-k mode: this chunk's summed pairs
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
    int bad = 0;
    const float* gl = reinterpret_cast<const float*>(glob_ptrs[rank]) + k.off;
    if (k.quant == 2) {
      // the chunk is one 4096-element block: add every sharer's (index, value) pairs
      __syncthreads();
      for (int i = threadIdx.x; i < kNvChunk; i += blockDim.x) dense[i] = 0.f;
      __syncthreads();
      const long long blk = (k.off + e0) / kNvChunk;
      for (int j = 0; j < k.nsh; ++j) {
        const uint16_t* si = reinterpret_cast<const uint16_t*>(qd_ptrs[k.sh[j]]) + blk * kcap;
        const float* sv = reinterpret_cast<const float*>(qs_ptrs[k.sh[j]]) + blk * kcap;
        for (int i = threadIdx.x; i < kcap; i += blockDim.x) {
          const uint16_t ix = *reinterpret_cast<const volatile uint16_t*>(si + i);
          if (ix != kSpEmpty && ix < kNvChunk) dense[ix] = __fadd_rn(dense[ix], *reinterpret_cast<const volatile float*>(sv + i));
        }
        __syncthreads();  // indices are unique within a sharer; sharers add in rank order
      }
    }
    // two float4 positions per thread and every sharer's load issued before any is used:
    // the peer loads cross NVLink, so the loads in flight, not the arithmetic, set the pace
    const long long stride = (long long)blockDim.x * 4;
    for (long long e = e0 + threadIdx.x * 4; e < e1; e += 2 * stride) {
      const long long ev[2] = {e, e + stride};
      const bool has[2] = {true, e + stride < e1};
      float4 acc[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k.quant == 2) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (has[u]) acc[u] = *reinterpret_cast<const float4*>(dense + (ev[u] - e0));
      } else {
        float4 d[2][kMaxSharers];
#pragma unroll
        for (int j = 0; j < kMaxSharers; ++j) {
          if (j >= k.nsh) break;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (!has[u]) continue;
            if (k.quant) {  // int4 codes + group scale of sharer j, dequantised in registers
              const long long ge = k.off + ev[u];
              const uint16_t c = *reinterpret_cast<const volatile uint16_t*>(
                  reinterpret_cast<const uint8_t*>(qd_ptrs[k.sh[j]]) + ge / 2);
              const float sc = *reinterpret_cast<const volatile float*>(
                  reinterpret_cast<const float*>(qs_ptrs[k.sh[j]]) + ge / kQGroup);
              d[u][j] = make_float4(__fmul_rn((float)((int)(c & 15u) - 8), sc),
                                    __fmul_rn((float)((int)((c >> 4) & 15u) - 8), sc),
                                    __fmul_rn((float)((int)((c >> 8) & 15u) - 8), sc),
                                    __fmul_rn((float)((int)((c >> 12) & 15u) - 8), sc));
            } else {
              d[u][j] = ld_cg4(reinterpret_cast<const float*>(delta_ptrs[k.sh[j]]) + k.off + ev[u]);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < kMaxSharers; ++j) {  // rank order: deterministic sums
          if (j >= k.nsh) break;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (!has[u]) continue;
            acc[u].x = __fadd_rn(acc[u].x, d[u][j].x);
            acc[u].y = __fadd_rn(acc[u].y, d[u][j].y);
            acc[u].z = __fadd_rn(acc[u].z, d[u][j].z);
            acc[u].w = __fadd_rn(acc[u].w, d[u][j].w);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!has[u]) continue;
        const long long eu = ev[u];
        const float4 gv = *reinterpret_cast<const float4*>(gl + eu);
        float4 mb = *reinterpret_cast<const float4*>(mom + k.off + eu);
        float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w}, g4[4] = {gv.x, gv.y, gv.z, gv.w};
        float b4[4] = {mb.x, mb.y, mb.z, mb.w}, n4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float dd = __fmul_rn(__fmul_rn(a4[i], k.inv_den), k.scale);
          if (!isfinite(dd)) {  // guard: a non-finite contribution leaves global and momentum as they are
            ++bad;
            n4[i] = g4[i];
            continue;
          }
          sq += dd * dd;
          const float b = first ? dd : __fadd_rn(__fmul_rn(b4[i], m), dd);
          b4[i] = b;
          const float upd = nesterov ? __fadd_rn(dd, __fmul_rn(m, b)) : b;
          n4[i] = __fadd_rn(g4[i], __fmul_rn(-lr, upd));
        }
        *reinterpret_cast<float4*>(mom + k.off + eu) = make_float4(b4[0], b4[1], b4[2], b4[3]);
        const float4 nv = make_float4(n4[0], n4[1], n4[2], n4[3]);
        for (int j = 0; j < k.nsh; ++j)
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(glob_ptrs[k.sh[j]]) + k.off + eu) = nv;
      }
    }
    outer_chunk_reduce(sq, bad, ch, sq_part, status);
  }
}

// After all ranks' peer stores: copy the fresh globals into this GPU's working copies
// (fp32 + bf16). One segment per module key with every local sharer, so each global is
// read once however many local paths use it.
__global__ void __launch_bounds__(256) outer_nvlink_bcast_kernel(const OuterSeg* __restrict__ segs, int nseg,
                                                                 const OuterLocal* __restrict__ locs,
                                                                 long long total_chunks,
                                                                 const unsigned long long* __restrict__ pads, int rank,
                                                                 int world, unsigned epoch, int* err,
                                                                 unsigned long long wait_ns) {
  if (!cross_gpu_barrier(pads, rank, world, 1, epoch, err, blockIdx.x == 0, wait_ns)) return;
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    const OuterSeg sg = segs[find_seg(segs, nseg, ch)];
    const long long e0 = (ch - sg.chunk0) * kOuterChunk;
    const long long e1 = min(e0 + kOuterChunk, sg.n);
    float sq = 0.f;
    int bad = 0;
    outer_chunk(sg, locs, e0, e1, 0.f, 0.f, 0, 0, sq, bad);
  }
}

}  // namespace odp

void outer_nvlink_apply(torch::Tensor keys, int64_t nkeys, int64_t total_chunks, torch::Tensor delta_ptrs,
                        torch::Tensor glob_ptrs, torch::Tensor pads, torch::Tensor mom, int64_t rank, int64_t world,
                        int64_t epoch, double lr, double m, bool nesterov, bool first, torch::Tensor sq_part,
                        torch::Tensor err, c10::optional<torch::Tensor> qd_ptrs, c10::optional<torch::Tensor> qs_ptrs,
                        int64_t kcap, c10::optional<torch::Tensor> status) {
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
      qs_ptrs.has_value() ? reinterpret_cast<const unsigned long long*>(qs_ptrs->data_ptr()) : nullptr, (int)kcap,
      odp::peer_wait_bound_ns(), status.has_value() ? status->data_ptr<int>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// regs: int64 [nregs][3] = (element offset (4096-aligned), true size, first block in
// launch order); spi / spv: [arena blocks][kcap] pair slots.
void outer_nvlink_topk(torch::Tensor regs, int64_t nregs, int64_t total_blocks, double density, int64_t kcap,
                       torch::Tensor delta, torch::Tensor res, torch::Tensor spi, torch::Tensor spv) {
  c10::cuda::CUDAGuard guard(delta.device());
  TORCH_CHECK(kcap >= 1 && kcap <= odp::kNvChunk, "outer_nvlink_topk: bad capacity");
  if (total_blocks == 0) return;
  odp::outer_nvlink_topk_kernel<<<(unsigned)total_blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::NvRegion*>(regs.data_ptr()), (int)nregs, density, (int)kcap,
      delta.data_ptr<float>(), res.data_ptr<float>(), reinterpret_cast<uint16_t*>(spi.data_ptr()),
      spv.data_ptr<float>());
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

// segs / locals: OuterSeg / OuterLocal tables (mode BCAST) of this GPU's shared keys.
void outer_nvlink_bcast(torch::Tensor segs, int64_t nseg, torch::Tensor locals, int64_t total_chunks,
                        torch::Tensor pads, int64_t rank, int64_t world, int64_t epoch, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(pads.device());
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  // always launched: every rank must take part in the barrier
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total_chunks, (int64_t)sms * 8));
  odp::outer_nvlink_bcast_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::OuterSeg*>(segs.data_ptr()), (int)nseg,
      reinterpret_cast<const odp::OuterLocal*>(locals.data_ptr()), total_chunks,
      reinterpret_cast<const unsigned long long*>(pads.data_ptr()), (int)rank, (int)world, (unsigned)epoch,
      err.data_ptr<int>(), odp::peer_wait_bound_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t outer_nvlink_chunk_elems() { return odp::kNvChunk; }

// Sets the bound of every later cross-GPU wait (outer step and intra-path data
// parallelism) in nanoseconds; 0 restores the 2 s default. Returns the previous bound.
int64_t set_peer_wait_ns(int64_t ns) {
  const int64_t old = (int64_t)odp::peer_wait_bound_ns();
  odp::peer_wait_bound_ns() = ns > 0 ? (unsigned long long)ns : odp::kWaitBoundNs;
  return old;
}
