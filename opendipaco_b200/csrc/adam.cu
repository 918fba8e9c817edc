// Inner-optimizer kernels over flat per-path buffers [G][P] (fp32).
//
// grad_clip: deterministic global-norm clip per path. Stage 1 writes per-block sums of
// squares; stage 2 sums them in a fixed order and stores
//     coef[g] = min(1, max_norm / (sqrt(sum) + 1e-6))
// (torch.nn.utils.clip_grad_norm_ semantics), which the update kernel folds into the
// gradient, so no extra pass over the gradients is spent on scaling.
//
// adamw: decoupled weight decay, bias-corrected moments, eps outside the sqrt
// (torch.optim.AdamW). Per-step scalars (lr, lr / (1 - b1^t), sqrt(1 - b2^t)) are read
// from a device array so a whole round of steps can live in one CUDA graph. Writes the
// fp32 master weight and its bf16 working copy for the GEMMs in the same pass.
//
// Skipped rows: both kernels can take the touched-row flags of one row-major region of
// every path (the embedding, whose backward writes only the rows of the batch's tokens):
// an element of an unflagged row counts as gradient 0, so the region needs no zeroing
// between steps. The gradient and the flag are loaded side by side and selected (a load
// that waited for the flag would double the latency chain of these memory-bound passes).
//
// adam8bit: blockwise 8-bit AdamW (blocks of 256): one warp per block dequantises m
// (int8, absmax / 127) and v (uint8 in the log domain: exp(q * scale + lo), floor
// 1e-20), updates in fp32 registers, requantises (round half to even) and updates the
// parameter from the unquantised moments -- a single pass over the state.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

// rows != nullptr: elements [r0, r0 + V * H) of each path are V rows of H; row v of path
// grp counts only when rows[grp * V + v] != 0.
struct RowSkip {
  const uint8_t* rows;
  long long r0;
  int H, V;
};

// True when the 4-element group at element i (i % 4 == 0, H % 4 == 0) lies in an unflagged row.
ODP_DEVICE bool row_skipped(const RowSkip& rs, int grp, long long i) {
  if (!rs.rows) return false;
  const long long d = i - rs.r0;
  if (d < 0 || d >= (long long)rs.V * rs.H) return false;
  // row = d / H without an integer division (this runs per 4 elements of a memory-bound
  // pass): d < 2^24 in practice is exact in fp32, and the estimate is fixed up by one step
  int r = __float2int_rz(__int2float_rn((int)d) * __frcp_rn((float)rs.H));
  const int di = (int)d;
  if (r * rs.H > di) --r;
  else if ((r + 1) * rs.H <= di) ++r;
  return rs.rows[(long long)grp * rs.V + r] == 0;
}

constexpr int kSqBlock = 256;
constexpr int kSqElemsPerBlock = 1 << 16;

__global__ void sumsq_kernel(const float* __restrict__ g, long long P, long long sg, int nblk, float* __restrict__ part,
                             RowSkip skip) {
  pdl_wait();
  pdl_trigger();
  const int grp = blockIdx.y, b = blockIdx.x;
  const float* base = g + grp * sg;
  const long long e0 = (long long)b * kSqElemsPerBlock;
  const long long e1 = min(e0 + kSqElemsPerBlock, P);
  float s = 0.f;
  for (long long i = e0 + threadIdx.x * 4; i < e1; i += kSqBlock * 4) {
    if (i + 4 <= e1) {
      float4 v = *reinterpret_cast<const float4*>(base + i);
      if (row_skipped(skip, grp, i)) v = make_float4(0.f, 0.f, 0.f, 0.f);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    } else {
      for (long long j = i; j < e1; ++j) s += base[j] * base[j];
    }
  }
  __shared__ float red[kSqBlock / 32];
  s = warp_sum(s);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kSqBlock / 32; ++w) t += red[w];
    part[(long long)grp * nblk + b] = t;
  }
}

__global__ void clip_coef_kernel(const float* __restrict__ part, int nblk, float max_norm, float* __restrict__ coef,
                                 float* __restrict__ norm_out) {
  pdl_wait();
  pdl_trigger();
  const int grp = blockIdx.x;
  __shared__ float red[256];
  float s = 0.f;
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) s += part[(long long)grp * nblk + i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float n = sqrtf(red[0]);
    if (norm_out) norm_out[grp] = n;
    coef[grp] = max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
  }
}

// Clip coefficient from sums of squares made by the gradients' producers: per path g,
// parts[g][0, nslot) (fp32 GEMM epilogues, one per 32 x 32 output box), esq[g][0, M)
// (embedding backward, one per written row) and the norm-weight gradients read directly
// (n_norm regions of H floats at offsets norm_offs within the path's gradient). One
// 256-thread block per path; fixed summation order.
__global__ void clip_coef_parts_kernel(const float* __restrict__ parts, long long nslot, const float* __restrict__ esq,
                                       int M, const float* __restrict__ grads, long long P,
                                       const long long* __restrict__ norm_offs, int n_norm, int H, float max_norm,
                                       float* __restrict__ coef, float* __restrict__ norm_out) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x;
  float s = 0.f;
  for (long long i = threadIdx.x; i < nslot; i += blockDim.x) s += parts[g * nslot + i];
  for (int i = threadIdx.x; i < M; i += blockDim.x) s += esq[(long long)g * M + i];
  for (int r = 0; r < n_norm; ++r) {
    const float* w = grads + g * P + norm_offs[r];
    for (int i = threadIdx.x; i < H; i += blockDim.x) s = fmaf(w[i], w[i], s);
  }
  __shared__ float red[256];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float n = sqrtf(red[0]);
    if (norm_out) norm_out[g] = n;
    coef[g] = max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
  }
}

// AdamW on four elements in registers (torch.optim.AdamW: decoupled decay, bias-corrected
// moments, eps outside the sqrt); the gradient is scaled by the clip coefficient first.
ODP_DEVICE void adamw4(float (&pv)[4], const float (&gv)[4], float (&mv)[4], float (&vv)[4], float cf, float decay,
                       float step_size, float bc2s, float b1, float b2, float eps) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float gr = gv[k] * cf;
    pv[k] *= decay;
    mv[k] = mv[k] + (1.f - b1) * (gr - mv[k]);
    vv[k] = vv[k] * b2 + (1.f - b2) * gr * gr;
    const float den = sqrtf(vv[k]) / bc2s + eps;
    pv[k] = pv[k] - step_size * (mv[k] / den);
  }
}

// sched: [G][4] = lr, step_size = lr / bc1, bc2_sqrt, active (0 -> leave this path untouched)
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ p16, long long P, long long sp,
                             long long s16, const float* __restrict__ coef, const float* __restrict__ sched, float b1,
                             float b2, float eps, float wd, RowSkip skip) {
  pdl_wait();
  pdl_trigger();
  const int grp = blockIdx.y;
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= P) return;
  const float* sc = sched + grp * 4;  // per path: lr, lr / bc1, sqrt(bc2), active
  if (sc[3] == 0.f) return;
  const float lr = sc[0], step_size = sc[1], bc2s = sc[2];
  const float cf = coef ? coef[grp] : 1.f;
  const float decay = 1.f - lr * wd;
  const long long o = grp * sp + i;
  const int n = (int)min((long long)4, P - i);
  float pv[4], gv[4], mv[4], vv[4];
  if (n == 4) {
    *reinterpret_cast<float4*>(pv) = *reinterpret_cast<const float4*>(p + o);
    const float4 gl = *reinterpret_cast<const float4*>(g + o);
    *reinterpret_cast<float4*>(gv) = row_skipped(skip, grp, i) ? make_float4(0.f, 0.f, 0.f, 0.f) : gl;
    *reinterpret_cast<float4*>(mv) = *reinterpret_cast<const float4*>(m + o);
    *reinterpret_cast<float4*>(vv) = *reinterpret_cast<const float4*>(v + o);
  } else {
    for (int k = 0; k < 4; ++k) {
      pv[k] = k < n ? p[o + k] : 0.f;
      gv[k] = k < n ? g[o + k] : 0.f;
      mv[k] = k < n ? m[o + k] : 0.f;
      vv[k] = k < n ? v[o + k] : 0.f;
    }
  }
  adamw4(pv, gv, mv, vv, cf, decay, step_size, bc2s, b1, b2, eps);
  if (n == 4) {
    *reinterpret_cast<float4*>(p + o) = *reinterpret_cast<float4*>(pv);
    *reinterpret_cast<float4*>(m + o) = *reinterpret_cast<float4*>(mv);
    *reinterpret_cast<float4*>(v + o) = *reinterpret_cast<float4*>(vv);
    uint2 w = make_uint2(pack_bf16(pv[0], pv[1]), pack_bf16(pv[2], pv[3]));
    *reinterpret_cast<uint2*>(p16 + grp * s16 + i) = w;
  } else {
    for (int k = 0; k < n; ++k) {
      p[o + k] = pv[k];
      m[o + k] = mv[k];
      v[o + k] = vv[k];
      p16[grp * s16 + i + k] = __float2bfloat16(pv[k]);
    }
  }
}

// ---------------------------------------------------------------- AdamW + pseudo-gradient
// AdamW for every path with one thread owning four elements of one region across all the
// paths (more independent loads per thread than one path per thread: measured 1.00 vs
// 0.89 of the HBM copy bandwidth at 16 paths). On the last inner step of a round the same
// pass also forms the outer step's pseudo-gradient partial sum_j w_j (global - new
// local_j) of every module key, so the outer step reads one partial per key instead of
// every local copy again.
//
// The path layout is cut into regions (a module's parameters sit at the same offsets in
// every path); region r lists (path, key) entries sorted by key and then path. A thread
// owns four consecutive elements of one region and walks its entries: AdamW for that
// path, then acc += w * (glob - new) -- the same fp32 operations in the same path order as
// the outer step's own accumulation -- storing acc into the key's pseudo-gradient buffer
// after the key's last entry. Private keys (one path) copy the new weight into the global.
struct AccRegion {
  long long begin, end;  // element range in every path's layout (begin % 4 == 0)
  int first, count;      // entries of this region (count <= kAccMaxEntries)
  long long cta0;        // first CTA of the region (each CTA covers kAccCtaElems elements of one region)
};
constexpr int kAccMaxEntries = 128;
constexpr int kAccCtaElems = 1024;
struct AccEntry {
  float* delta;  // key's pseudo-gradient buffer at the region start (null: private key)
  float* glob;   // key's global buffer at the region start
  int g;         // path
  int flags;     // 1: last entry of its key in this region
  float weight;
  int pad;
};

// Every CTA lies in one region: its entries, their schedules and clip coefficients are
// staged in shared memory once, so a thread's loads of a path's state wait on nothing
// but their own addresses. Entries are handled two at a time, every load of both paths
// issued before either's stores (stores through the same base pointers would otherwise
// keep the compiler from moving the next path's loads ahead of them).
constexpr int kAccBatch = 2;

__global__ void __launch_bounds__(256) adamw_acc_kernel(
    float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
    __nv_bfloat16* __restrict__ p16, long long sp, long long s16, const float* __restrict__ coef,
    const float* __restrict__ sched, float b1, float b2, float eps, float wd, RowSkip skip,
    const AccRegion* __restrict__ regs, int nregs, const AccEntry* __restrict__ ents, int accumulate) {
  pdl_wait();
  pdl_trigger();
  __shared__ AccRegion sR;
  __shared__ AccEntry sE[kAccMaxEntries];
  __shared__ float4 sS[kAccMaxEntries];  // lr, lr / bc1, sqrt(bc2), active of the entry's path
  __shared__ float sC[kAccMaxEntries];   // clip coefficient of the entry's path
  if (threadIdx.x == 0) {
    int lo = 0, hi = nregs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (regs[mid].cta0 <= (long long)blockIdx.x) lo = mid;
      else hi = mid - 1;
    }
    sR = regs[lo];
  }
  __syncthreads();
  const AccRegion R = sR;
  for (int k = threadIdx.x; k < R.count; k += blockDim.x) {
    const AccEntry e = ents[R.first + k];
    sE[k] = e;
    sS[k] = *reinterpret_cast<const float4*>(sched + e.g * 4);
    sC[k] = coef ? coef[e.g] : 1.f;
  }
  __syncthreads();
  const long long off = (blockIdx.x - R.cta0) * kAccCtaElems + threadIdx.x * 4;
  const long long i = R.begin + off;
  if (i >= R.end) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 gl = make_float4(0.f, 0.f, 0.f, 0.f);
  bool have_glob = false;
  for (int k0 = 0; k0 < R.count; k0 += kAccBatch) {
    float pv[kAccBatch][4], gv[kAccBatch][4], mv[kAccBatch][4], vv[kAccBatch][4];
#pragma unroll
    for (int u = 0; u < kAccBatch; ++u) {
      if (k0 + u >= R.count) continue;
      const int grp = sE[k0 + u].g;
      const long long o = grp * sp + i;
      *reinterpret_cast<float4*>(pv[u]) = *reinterpret_cast<const float4*>(p + o);
      if (sS[k0 + u].w != 0.f) {
        const float4 gr = *reinterpret_cast<const float4*>(g + o);
        *reinterpret_cast<float4*>(gv[u]) = row_skipped(skip, grp, i) ? make_float4(0.f, 0.f, 0.f, 0.f) : gr;
        *reinterpret_cast<float4*>(mv[u]) = *reinterpret_cast<const float4*>(m + o);
        *reinterpret_cast<float4*>(vv[u]) = *reinterpret_cast<const float4*>(v + o);
      }
    }
#pragma unroll
    for (int u = 0; u < kAccBatch; ++u) {
      if (k0 + u >= R.count) break;
      const AccEntry& E = sE[k0 + u];
      const float4 sc = sS[k0 + u];
      if (sc.w != 0.f) {
        const long long o = E.g * sp + i;
        adamw4(pv[u], gv[u], mv[u], vv[u], sC[k0 + u], 1.f - sc.x * wd, sc.y, sc.z, b1, b2, eps);
        *reinterpret_cast<float4*>(p + o) = *reinterpret_cast<float4*>(pv[u]);
        *reinterpret_cast<float4*>(m + o) = *reinterpret_cast<float4*>(mv[u]);
        *reinterpret_cast<float4*>(v + o) = *reinterpret_cast<float4*>(vv[u]);
        *reinterpret_cast<uint2*>(p16 + E.g * s16 + i) =
            make_uint2(pack_bf16(pv[u][0], pv[u][1]), pack_bf16(pv[u][2], pv[u][3]));
      }
      if (!accumulate) continue;  // an inner step that is not the round's last
      if (E.delta == nullptr) {  // private key: the global is the path's own copy
        *reinterpret_cast<float4*>(E.glob + off) = *reinterpret_cast<float4*>(pv[u]);
        continue;
      }
      if (!have_glob) {
        gl = *reinterpret_cast<const float4*>(E.glob + off);
        have_glob = true;
      }
      const float w = E.weight;
      acc.x = __fadd_rn(acc.x, __fmul_rn(w, __fsub_rn(gl.x, pv[u][0])));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w, __fsub_rn(gl.y, pv[u][1])));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w, __fsub_rn(gl.z, pv[u][2])));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w, __fsub_rn(gl.w, pv[u][3])));
      if (E.flags & 1) {
        *reinterpret_cast<float4*>(E.delta + off) = acc;
        acc = make_float4(0.f, 0.f, 0.f, 0.f);
        have_glob = false;
      }
    }
  }
}

// ---------------------------------------------------------------- 8-bit Adam
// One warp per 256-element block (8 consecutive elements per lane). With `vec` (every base
// 16-byte aligned, codes 8-byte aligned) a lane issues all of its loads up front as
// vectors -- two float4 of gradient, two of weights, 8 bytes of each code -- so a warp has
// its whole block in flight before the block reductions; the arithmetic per element is the
// same in both forms.
template <bool VEC>
ODP_DEVICE void a8_load(const float* __restrict__ src, long long e0, long long n, float (&v)[8]) {
  if (VEC) {
    const float4 a = *reinterpret_cast<const float4*>(src + e0), b = *reinterpret_cast<const float4*>(src + e0 + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = e0 + k < n ? src[e0 + k] : 0.f;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256, 4) adam8bit_kernel(float* __restrict__ p, const float* __restrict__ g, long long n,
                                                       int8_t* __restrict__ mq, float* __restrict__ mabs,
                                                       uint8_t* __restrict__ vq, float* __restrict__ vlo,
                                                       float* __restrict__ vsc, long long nblocks,
                                                       long long blocks_per_group, const float* __restrict__ coef,
                                                       const float* __restrict__ sched, float b1, float b2, float eps,
                                                       float wd, int first, __nv_bfloat16* __restrict__ p16) {
  pdl_wait();
  pdl_trigger();
  const long long blk = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (blk >= nblocks) return;
  const long long grp = blocks_per_group > 0 ? blk / blocks_per_group : 0;
  const float* scd = sched + grp * 4;  // per path: lr, lr / bc1, sqrt(bc2), active
  if (scd[3] == 0.f) return;
  const long long e0 = blk * 256 + lane * 8;
  const bool full = VEC && e0 + 8 <= n;
  float gv[8], pv[8];
  int8_t mc[8];
  uint8_t vc[8];
  if (full) {
    a8_load<true>(g, e0, n, gv);
    a8_load<true>(p, e0, n, pv);
    *reinterpret_cast<uint2*>(mc) = *reinterpret_cast<const uint2*>(mq + e0);
    *reinterpret_cast<uint2*>(vc) = *reinterpret_cast<const uint2*>(vq + e0);
  } else {
    a8_load<false>(g, e0, n, gv);
    a8_load<false>(p, e0, n, pv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mc[k] = mq[e0 + k];
      vc[k] = vq[e0 + k];
    }
  }
  const float lr = scd[0], step_size = scd[1], bc2s = scd[2];
  const bool first_step = first || scd[3] > 1.5f;  // 2.0 marks a path's first step
  const float cf = coef ? coef[grp] : 1.f;
  const float mscale = mabs[blk] / 127.f;
  const float lo = vlo[blk], sc = vsc[blk];
  float mv[8], vv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    gv[k] = e0 + k < n ? gv[k] * cf : 0.f;
    mv[k] = (float)mc[k] * mscale;
    vv[k] = first_step ? 0.f : __expf((float)vc[k] * sc + lo);
    mv[k] = mv[k] * b1 + (1.f - b1) * gv[k];
    vv[k] = vv[k] * b2 + (1.f - b2) * gv[k] * gv[k];
  }
  // requantise m: symmetric absmax; v: log domain over the block's range
  float amax = 0.f, lmin = INFINITY, lmax = -INFINITY;
  float lv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    amax = fmaxf(amax, fabsf(mv[k]));
    lv[k] = __logf(fmaxf(vv[k], 1e-20f));
    lmin = fminf(lmin, lv[k]);
    lmax = fmaxf(lmax, lv[k]);
  }
  amax = warp_max(amax);
  lmax = warp_max(lmax);
  lmin = -warp_max(-lmin);
  const float qs = amax > 0.f ? amax / 127.f : 1.f;
  const float vs = fmaxf((lmax - lmin) / 255.f, 1e-12f);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    mc[k] = (int8_t)fminf(fmaxf(rintf(mv[k] / qs), -127.f), 127.f);
    vc[k] = (uint8_t)fminf(fmaxf(rintf((lv[k] - lmin) / vs), 0.f), 255.f);
  }
  if (lane == 0) {
    mabs[blk] = amax;
    vlo[blk] = lmin;
    vsc[blk] = vs;
  }
  const float decay = 1.f - lr * wd;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float den = sqrtf(vv[k]) / bc2s + eps;
    pv[k] = pv[k] * decay - step_size * (mv[k] / den);
  }
  if (full) {
    *reinterpret_cast<uint2*>(mq + e0) = *reinterpret_cast<const uint2*>(mc);
    *reinterpret_cast<uint2*>(vq + e0) = *reinterpret_cast<const uint2*>(vc);
    *reinterpret_cast<float4*>(p + e0) = make_float4(pv[0], pv[1], pv[2], pv[3]);
    *reinterpret_cast<float4*>(p + e0 + 4) = make_float4(pv[4], pv[5], pv[6], pv[7]);
    if (p16)
      *reinterpret_cast<uint4*>(p16 + e0) = make_uint4(pack_bf16(pv[0], pv[1]), pack_bf16(pv[2], pv[3]),
                                                       pack_bf16(pv[4], pv[5]), pack_bf16(pv[6], pv[7]));
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mq[e0 + k] = mc[k];
      vq[e0 + k] = vc[k];
      if (e0 + k < n) {
        p[e0 + k] = pv[k];
        if (p16) p16[e0 + k] = __float2bfloat16(pv[k]);
      }
    }
  }
}

}  // namespace odp

static odp::RowSkip row_skip(const c10::optional<torch::Tensor>& rows, int64_t r0, int64_t H, int64_t V) {
  odp::RowSkip s{nullptr, 0, 1, 0};
  if (rows.has_value()) {
    TORCH_CHECK(rows->scalar_type() == at::kByte && H % 4 == 0 && r0 % 4 == 0, "row flags: uint8, H and r0 % 4 == 0");
    s = odp::RowSkip{rows->data_ptr<uint8_t>(), r0, (int)H, (int)V};
  }
  return s;
}

void grad_clip_coef(torch::Tensor grads, int64_t P, int64_t sg, int64_t G, double max_norm, torch::Tensor work,
                    torch::Tensor coef, c10::optional<torch::Tensor> norm_out, c10::optional<torch::Tensor> rows,
                    int64_t r0, int64_t H, int64_t V) {
  c10::cuda::CUDAGuard guard(grads.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int nblk = (int)((P + odp::kSqElemsPerBlock - 1) / odp::kSqElemsPerBlock);
  TORCH_CHECK(work.numel() >= G * nblk, "grad_clip_coef: work buffer too small");
  C10_CUDA_CHECK(odp::launch_pdl((odp::sumsq_kernel), dim3(dim3(nblk, (unsigned)G)), dim3(odp::kSqBlock), 0, st, grads.data_ptr<float>(), P, sg, nblk,
                                                                      work.data_ptr<float>(), row_skip(rows, r0, H, V)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  C10_CUDA_CHECK(odp::launch_pdl((odp::clip_coef_kernel), dim3((unsigned)G), dim3(256), 0, st, work.data_ptr<float>(), nblk, (float)max_norm,
                                                      coef.data_ptr<float>(),
                                                      norm_out.has_value() ? norm_out->data_ptr<float>() : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void grad_clip_coef_parts(torch::Tensor parts, int64_t nslot, torch::Tensor esq, int64_t M, torch::Tensor grads,
                          int64_t P, torch::Tensor norm_offs, int64_t H, int64_t G, double max_norm, torch::Tensor coef,
                          c10::optional<torch::Tensor> norm_out) {
  c10::cuda::CUDAGuard guard(grads.device());
  TORCH_CHECK(parts.numel() >= G * nslot && esq.numel() >= G * M, "grad_clip_coef_parts: partials too small");
  C10_CUDA_CHECK(odp::launch_pdl((odp::clip_coef_parts_kernel), dim3((unsigned)G), dim3(256), 0, at::cuda::getCurrentCUDAStream(), parts.data_ptr<float>(), nslot, esq.data_ptr<float>(), (int)M, grads.data_ptr<float>(), P,
      reinterpret_cast<const long long*>(norm_offs.data_ptr<int64_t>()), (int)norm_offs.numel(), (int)H,
      (float)max_norm, coef.data_ptr<float>(), norm_out.has_value() ? norm_out->data_ptr<float>() : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor p16, int64_t P,
                int64_t sp, int64_t s16, int64_t G, c10::optional<torch::Tensor> coef, torch::Tensor sched, double b1,
                double b2, double eps, double wd, c10::optional<torch::Tensor> rows, int64_t r0, int64_t H,
                int64_t V) {
  c10::cuda::CUDAGuard guard(p.device());
  TORCH_CHECK(P % 4 == 0 || G == 1, "adamw_step: per-group length must be a multiple of 4");
  const long long threads = (P + 3) / 4;
  dim3 grid((unsigned)((threads + 255) / 256), (unsigned)G);
  C10_CUDA_CHECK(odp::launch_pdl((odp::adamw_kernel), dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream(), p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(p16.data_ptr()), P, sp, s16,
      coef.has_value() ? coef->data_ptr<float>() : nullptr, sched.data_ptr<float>(), (float)b1, (float)b2,
      (float)eps, (float)wd, row_skip(rows, r0, H, V)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// AdamW over every path of the layout, one region per CTA; with `accumulate` (the last
// inner step of a round) fused with the outer pseudo-gradient accumulation.
// regions: int64 [nregs, 4] AccRegion records (their CTAs, kAccCtaElems elements each, in
// region order: ctas = total CTA count); entries: int64 [nents, 4] AccEntry records.
// Regions begin at multiples of 4 elements; buffers are 16-byte aligned.
void adamw_acc_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor p16, int64_t ctas,
                    int64_t sp, int64_t s16, c10::optional<torch::Tensor> coef, torch::Tensor sched, double b1,
                    double b2, double eps, double wd, c10::optional<torch::Tensor> rows, int64_t r0, int64_t H,
                    int64_t V, torch::Tensor regions, int64_t nregs, torch::Tensor entries, bool accumulate) {
  static_assert(sizeof(odp::AccRegion) == 32 && sizeof(odp::AccEntry) == 32, "AccRegion / AccEntry layout");
  c10::cuda::CUDAGuard guard(p.device());
  TORCH_CHECK(sp % 4 == 0 && s16 % 4 == 0, "adamw_acc_step: strides must be multiples of 4");
  TORCH_CHECK(regions.is_cuda() && entries.is_cuda() && nregs >= 1 && ctas >= 1, "adamw_acc_step: tables on the device");
  TORCH_CHECK(odp::kAccCtaElems == 256 * 4, "adamw_acc_step: one CTA covers 256 x 4 elements");
  C10_CUDA_CHECK(odp::launch_pdl((odp::adamw_acc_kernel), dim3((unsigned)ctas), dim3(256), 0, at::cuda::getCurrentCUDAStream(), p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(p16.data_ptr()), sp, s16,
      coef.has_value() ? coef->data_ptr<float>() : nullptr, sched.data_ptr<float>(), (float)b1, (float)b2,
      (float)eps, (float)wd, row_skip(rows, r0, H, V), reinterpret_cast<const odp::AccRegion*>(regions.data_ptr()),
      (int)nregs, reinterpret_cast<const odp::AccEntry*>(entries.data_ptr()), accumulate ? 1 : 0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adam8bit_step(torch::Tensor p, torch::Tensor g, torch::Tensor mq, torch::Tensor mabs, torch::Tensor vq,
                   torch::Tensor vlo, torch::Tensor vsc, c10::optional<torch::Tensor> coef, torch::Tensor sched,
                   double b1, double b2, double eps, double wd, bool first, c10::optional<torch::Tensor> p16,
                   int64_t blocks_per_group) {
  c10::cuda::CUDAGuard guard(p.device());
  const long long n = p.numel(), nb = mabs.numel();
  TORCH_CHECK(mq.numel() == nb * 256 && vq.numel() == nb * 256, "adam8bit_step: state must be [nblocks, 256]");
  TORCH_CHECK(nb * 256 >= n, "adam8bit_step: too few blocks");
  const long long threads = nb * 32;
  auto al = [](const void* q, int a) { return reinterpret_cast<uintptr_t>(q) % a == 0; };
  const bool vec = al(p.data_ptr(), 16) && al(g.data_ptr(), 16) && al(mq.data_ptr(), 8) && al(vq.data_ptr(), 8) &&
                   (!p16.has_value() || al(p16->data_ptr(), 16));
  auto kern = vec ? odp::adam8bit_kernel<true> : odp::adam8bit_kernel<false>;
  C10_CUDA_CHECK(odp::launch_pdl(kern, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0,
                                 at::cuda::getCurrentCUDAStream(), p.data_ptr<float>(), g.data_ptr<float>(), n,
                                 mq.data_ptr<int8_t>(), mabs.data_ptr<float>(), vq.data_ptr<uint8_t>(),
                                 vlo.data_ptr<float>(), vsc.data_ptr<float>(), nb, blocks_per_group,
                                 coef.has_value() ? coef->data_ptr<float>() : nullptr, sched.data_ptr<float>(),
                                 (float)b1, (float)b2, (float)eps, (float)wd, first ? 1 : 0,
                                 p16.has_value() ? reinterpret_cast<__nv_bfloat16*>(p16->data_ptr()) : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
