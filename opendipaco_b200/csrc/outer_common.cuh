// The DiLoCo outer-step arithmetic over one 4096-element chunk of a module, shared by
// the single-GPU outer step (outer.cu) and the cross-GPU broadcast (outer_nvlink.cu).
//
// A segment is one module key: its flat fp32 global buffer, momentum, pseudo-gradient
// buffer and the working copies of the paths on this GPU that use it (fp32 master + bf16
// GEMM copy, with their outer weights). Per element e, by mode:
//   OUTER  acc = sum_j w_j (glob[e] - local_j[e])        (path order, fp32, no FMA)
//          d = acc * inv_den * scale
//          buf = first ? d : m buf + d ;  upd = nesterov ? d + m buf : buf
//          glob[e] -= lr upd ; every local_j[e] = glob[e] (fp32 + bf16)
//   ACC    delta[e] = acc                                 (the partial of the cross-GPU step)
//   APPLY  OUTER with acc = delta[e] (the pseudo-gradient was accumulated earlier, by the
//          ACC mode or by the last inner step's optimizer kernel)
//   COPY   glob[e] = local_0[e]                            (private module: no outer step)
//   BCAST  every local_j[e] = glob[e]
// Guard: an element whose d is not finite (a diverged path's NaN / Inf) is not applied:
// global and momentum keep their values, the working copies are reset to the global, and
// the element is counted in the caller's status word. Squares of the applied d are summed
// per chunk for the delta-norm metric.
//
// Every buffer is 16-byte aligned and every segment a multiple of 4 elements (the host
// pads module regions to 256 elements), so each thread moves float4 / 4 x bf16 groups;
// the working copies of up to four paths are loaded before any is used, so a thread keeps
// several independent loads in flight.
#pragma once

#include "common.cuh"

namespace odp {

struct OuterSeg {
  float* glob;
  float* mom;       // null for COPY / BCAST
  float* delta;     // ACC writes, APPLY reads
  long long n;      // elements (multiple of 4)
  int first_local;  // index into the local table
  int nlocal;
  int mode;
  float scale;      // sqrt(sharing) (or 1)
  float inv_den;    // 1 / sum of weights (normalize) or 1
  long long chunk0; // first chunk of this segment in the flat chunk space
};

struct OuterLocal {
  float* w32;
  __nv_bfloat16* w16;
  float weight;
};

enum OuterMode : int { OUTER_STEP = 0, OUTER_COPY = 1, OUTER_BCAST = 2, OUTER_ACC = 3, OUTER_APPLY = 4 };

constexpr int kOuterChunk = 4096;

ODP_DEVICE int find_seg(const OuterSeg* __restrict__ segs, int nseg, long long ch) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (segs[mid].chunk0 <= ch) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

ODP_DEVICE void store_locals4(const OuterLocal* __restrict__ locs, int first, int n, long long e, float4 v) {
  const uint2 h = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
  for (int j = 0; j < n; ++j) {
    const OuterLocal L = locs[first + j];
    *reinterpret_cast<float4*>(L.w32 + e) = v;
    if (L.w16) *reinterpret_cast<uint2*>(L.w16 + e) = h;
  }
}

ODP_DEVICE float4 fadd4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// acc = sum_j w_j (g - local_j) over the segment's locals, in order.
ODP_DEVICE float4 pseudo_grad4(const OuterLocal* __restrict__ locs, int first, int n, long long e, float4 g) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = 0; j0 < n; j0 += 4) {
    float4 l[4];
    float w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j0 + u < n) {
        const OuterLocal L = locs[first + j0 + u];
        l[u] = *reinterpret_cast<const float4*>(L.w32 + e);
        w[u] = L.weight;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j0 + u >= n) break;
      acc.x = __fadd_rn(acc.x, __fmul_rn(w[u], __fsub_rn(g.x, l[u].x)));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w[u], __fsub_rn(g.y, l[u].y)));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w[u], __fsub_rn(g.z, l[u].z)));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w[u], __fsub_rn(g.w, l[u].w)));
    }
  }
  return acc;
}

// One element of the outer update; returns the new global. `bad` counts skipped elements.
ODP_DEVICE float outer_update1(float acc, float g, float& buf, const OuterSeg& s, float lr, float m, int nesterov,
                               int first, float& sq, int& bad) {
  const float d = __fmul_rn(__fmul_rn(acc, s.inv_den), s.scale);
  if (!isfinite(d)) {
    ++bad;
    return g;
  }
  sq += d * d;
  const float b = first ? d : __fadd_rn(__fmul_rn(buf, m), d);
  buf = b;
  const float upd = nesterov ? __fadd_rn(d, __fmul_rn(m, b)) : b;
  return __fadd_rn(g, __fmul_rn(-lr, upd));
}

// Process elements [e0, e1) of segment s (e0, e1 multiples of 4) with the CTA's threads.
ODP_DEVICE void outer_chunk(const OuterSeg& s, const OuterLocal* __restrict__ locs, long long e0, long long e1,
                            float lr, float m, int nesterov, int first, float& sq, int& bad) {
  for (long long e = e0 + (long long)threadIdx.x * 4; e < e1; e += (long long)blockDim.x * 4) {
    if (s.mode == OUTER_COPY) {
      *reinterpret_cast<float4*>(s.glob + e) = *reinterpret_cast<const float4*>(locs[s.first_local].w32 + e);
      continue;
    }
    const float4 g = *reinterpret_cast<const float4*>(s.glob + e);
    if (s.mode == OUTER_BCAST) {
      store_locals4(locs, s.first_local, s.nlocal, e, g);
      continue;
    }
    float4 acc;
    if (s.mode == OUTER_APPLY) {
      acc = *reinterpret_cast<const float4*>(s.delta + e);
    } else {
      acc = pseudo_grad4(locs, s.first_local, s.nlocal, e, g);
      if (s.mode == OUTER_ACC) {
        *reinterpret_cast<float4*>(s.delta + e) = acc;
        continue;
      }
    }
    float4 b = *reinterpret_cast<const float4*>(s.mom + e);
    float4 ng;
    ng.x = outer_update1(acc.x, g.x, b.x, s, lr, m, nesterov, first, sq, bad);
    ng.y = outer_update1(acc.y, g.y, b.y, s, lr, m, nesterov, first, sq, bad);
    ng.z = outer_update1(acc.z, g.z, b.z, s, lr, m, nesterov, first, sq, bad);
    ng.w = outer_update1(acc.w, g.w, b.w, s, lr, m, nesterov, first, sq, bad);
    *reinterpret_cast<float4*>(s.mom + e) = b;
    *reinterpret_cast<float4*>(s.glob + e) = ng;
    store_locals4(locs, s.first_local, s.nlocal, e, ng);
  }
}

// CTA-wide: sq_part[ch] = sum of the threads' sq (fixed order); status += sum of bad.
ODP_DEVICE void outer_chunk_reduce(float sq, int bad, long long ch, float* sq_part, int* status) {
  __shared__ float red[32];
  __shared__ int nbad;
  if (threadIdx.x == 0) nbad = 0;
  sq = warp_sum(sq);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sq;
  if (bad) atomicAdd(&nbad, bad);
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) t += red[w];
    if (sq_part) sq_part[ch] = t;
    if (nbad && status) atomicAdd(status, nbad);
  }
  __syncthreads();
}

}  // namespace odp
