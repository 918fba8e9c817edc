// RMSNorm and token-embedding kernels (grouped over G paths).
//
// RMSNorm (HF Llama semantics, fp32 math): y = w * (x * rsqrt(mean(x^2) + eps)),
// emitted as bf16 for the following GEMM, plus the per-row rstd for backward.
// Backward: dx = rstd * (w*dy - xhat * mean(w*dy*xhat)) (+ incoming residual grad),
// dw = sum_rows dy * xhat via per-block partials reduced in a fixed order (no
// float atomics, so results are bitwise reproducible run to run).
//
// Embedding backward is deterministic too: for every token row r whose id has no
// earlier occurrence in the batch, one warp sums dx over all rows with that id in
// increasing row order and writes dE[id]. Rows of ids absent from the batch are
// left untouched (the caller zeroes the gradient buffer once per step).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

// x: [G][M][H] fp32 (row stride H, group stride sx); w: [G] x H fp32 at group stride sw.
// One warp per row; H % 128 == 0 (float4 per lane per step).
__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, long long sx, const float* __restrict__ w,
                                   long long sw, __nv_bfloat16* __restrict__ y, long long sy,
                                   float* __restrict__ rstd, int M, int H, int G, float eps) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= G * M) return;
  const int g = warp / M, r = warp % M;
  const float4* xr = reinterpret_cast<const float4*>(x + g * sx + (long long)r * H);
  const float4* wr = reinterpret_cast<const float4*>(w + g * sw);
  float ss = 0.f;
  for (int i = lane; i < H / 4; i += 32) {
    float4 v = xr[i];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / H + eps);
  uint2* yr = reinterpret_cast<uint2*>(y + g * sy + (long long)r * H);
  for (int i = lane; i < H / 4; i += 32) {
    float4 v = xr[i], ww = wr[i];
    yr[i] = make_uint2(pack_bf16(ww.x * (v.x * rs), ww.y * (v.y * rs)), pack_bf16(ww.z * (v.z * rs), ww.w * (v.w * rs)));
  }
  if (lane == 0) rstd[(long long)g * M + r] = rs;
}

// The same with the row held in registers (H = 128 * NV): x is read once, the weights
// once per warp, and four rows are in flight per warp.
template <int NV, int R>
__global__ void __launch_bounds__(256) rmsnorm_fwd_reg_kernel(const float* __restrict__ x, long long sx,
                                                              const float* __restrict__ w, long long sw,
                                                              __nv_bfloat16* __restrict__ y, long long sy,
                                                              float* __restrict__ rstd, int M, int H, int G,
                                                              float eps) {
  pdl_wait();
  pdl_trigger();
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32 * R;
  const int lane = threadIdx.x % 32;
  float4 v[R][NV];
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const long long wr_ = warp0 + k;
    if (wr_ >= (long long)G * M) break;
    const int g = (int)(wr_ / M), r = (int)(wr_ % M);
    const float4* xr = reinterpret_cast<const float4*>(x + g * sx + (long long)r * H);
#pragma unroll
    for (int j = 0; j < NV; ++j) v[k][j] = xr[lane + 32 * j];
  }
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const long long wr_ = warp0 + k;
    if (wr_ >= (long long)G * M) break;
    const int g = (int)(wr_ / M), r = (int)(wr_ % M);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) ss += v[k][j].x * v[k][j].x + v[k][j].y * v[k][j].y + v[k][j].z * v[k][j].z + v[k][j].w * v[k][j].w;
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / H + eps);
    const float4* wr = reinterpret_cast<const float4*>(w + g * sw);
    uint2* yr = reinterpret_cast<uint2*>(y + g * sy + (long long)r * H);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 ww = wr[lane + 32 * j], a = v[k][j];
      yr[lane + 32 * j] = make_uint2(pack_bf16(ww.x * (a.x * rs), ww.y * (a.y * rs)),
                                     pack_bf16(ww.z * (a.z * rs), ww.w * (a.w * rs)));
    }
    if (lane == 0) rstd[(long long)g * M + r] = rs;
  }
}

// dy: [G][M][H] fp32 (grad w.r.t. the norm output); dres: optional residual grad added to dx.
// dx may alias dres. dw_part: [G][nblk][H] partial sums of dy*xhat for rows of each block.
constexpr int kNormRowsPerBlock = 32;

__global__ void rmsnorm_bwd_kernel(const float* __restrict__ x, long long sx, const float* __restrict__ w,
                                   long long sw, const float* __restrict__ rstd, const float* __restrict__ dy,
                                   long long sdy, const float* dres, float* dx, long long sdx,
                                   __nv_bfloat16* dx16, float* __restrict__ dw_part, int M, int H, int G,
                                   int rpb) {
  pdl_wait();
  pdl_trigger();
  // block = 256 threads = 8 warps; block handles kNormRowsPerBlock rows of one group
  const int nblk = (M + rpb - 1) / rpb;
  const int g = blockIdx.x / nblk, b = blockIdx.x % nblk;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  extern __shared__ float sdw[];  // [8 warps][H]
  for (int i = threadIdx.x; i < 8 * H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  const float* wg = w + g * sw;
  const int n4 = H / 4;  // float4 columns (H % 128 == 0: n4 is a multiple of 32)
  for (int rr = warp; rr < rpb; rr += 8) {
    const int r = b * rpb + rr;
    if (r >= M) break;
    const float4* xr = reinterpret_cast<const float4*>(x + g * sx + (long long)r * H);
    const float4* dyr = reinterpret_cast<const float4*>(dy + g * sdy + (long long)r * H);
    const float4* w4 = reinterpret_cast<const float4*>(wg);
    const float rs = rstd[(long long)g * M + r];
    float dot = 0.f;
    for (int i = lane; i < n4; i += 32) {
      const float4 a = w4[i], d = dyr[i], xv = xr[i];
      dot += a.x * d.x * (xv.x * rs) + a.y * d.y * (xv.y * rs) + a.z * d.z * (xv.z * rs) + a.w * d.w * (xv.w * rs);
    }
    dot = warp_sum(dot) / H;
    float4* dxr = reinterpret_cast<float4*>(dx + g * sdx + (long long)r * H);
    const float4* drr = dres ? reinterpret_cast<const float4*>(dres + g * sdx + (long long)r * H) : nullptr;
    uint2* d16 = dx16 ? reinterpret_cast<uint2*>(dx16 + g * sdx + (long long)r * H) : nullptr;
    float4* acc = reinterpret_cast<float4*>(sdw + warp * H);
    for (int i = lane; i < n4; i += 32) {
      const float4 a = w4[i], d = dyr[i], xv = xr[i];
      const float4 xh = make_float4(xv.x * rs, xv.y * rs, xv.z * rs, xv.w * rs);
      float4 v = make_float4(rs * (a.x * d.x - xh.x * dot), rs * (a.y * d.y - xh.y * dot),
                             rs * (a.z * d.z - xh.z * dot), rs * (a.w * d.w - xh.w * dot));
      if (drr) {
        const float4 q = drr[i];
        v.x += q.x;
        v.y += q.y;
        v.z += q.z;
        v.w += q.w;
      }
      dxr[i] = v;
      if (d16) d16[i] = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
      float4 t = acc[i];
      t.x += d.x * xh.x;
      t.y += d.y * xh.y;
      t.z += d.z * xh.z;
      t.w += d.w * xh.w;
      acc[i] = t;
    }
  }
  __syncthreads();
  float* out = dw_part + ((long long)g * nblk + b) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += sdw[k * H + i];
    out[i] = s;
  }
}

// Register-resident variant (H = 128 * NV): each warp loads its row's x, dy and residual
// grad once, keeps the weights and its dw partial in registers, and folds the partials of
// its block's 8 warps in a fixed order at the end. Same arithmetic as rmsnorm_bwd_kernel.
// Up to H = 384 the row fits in 80 registers, so three blocks (24 warps) share an SM
// instead of two; wider rows keep the compiler's own register count.
template <int NV>
__global__ void __launch_bounds__(256, (NV <= 3) ? 3 : 1)
    rmsnorm_bwd_reg_kernel(const float* __restrict__ x, long long sx,
                                                              const float* __restrict__ w, long long sw,
                                                              const float* __restrict__ rstd,
                                                              const float* __restrict__ dy, long long sdy,
                                                              const float* dres, float* dx, long long sdx,
                                                              __nv_bfloat16* dx16, float* __restrict__ dw_part, int M,
                                                              int H, int G, int rpb) {
  pdl_wait();
  pdl_trigger();
  const int nblk = (M + rpb - 1) / rpb;
  const int g = blockIdx.x / nblk, b = blockIdx.x % nblk;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  extern __shared__ float sdw[];  // [8 warps][H]
  const float4* w4 = reinterpret_cast<const float4*>(w + g * sw);
  float4 wv[NV], acc[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    wv[j] = w4[lane + 32 * j];
    acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll 1
  for (int rr = warp; rr < rpb; rr += 8) {
    const int r = b * rpb + rr;
    if (r >= M) break;
    const float4* xr = reinterpret_cast<const float4*>(x + g * sx + (long long)r * H);
    const float4* dyr = reinterpret_cast<const float4*>(dy + g * sdy + (long long)r * H);
    const float4* drr = dres ? reinterpret_cast<const float4*>(dres + g * sdx + (long long)r * H) : nullptr;
    float4 d[NV], xv[NV], q[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      d[j] = dyr[lane + 32 * j];
      xv[j] = xr[lane + 32 * j];
      q[j] = drr ? drr[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float rs = rstd[(long long)g * M + r];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 a = wv[j], dd = d[j], xx = xv[j];
      dot += a.x * dd.x * (xx.x * rs) + a.y * dd.y * (xx.y * rs) + a.z * dd.z * (xx.z * rs) + a.w * dd.w * (xx.w * rs);
    }
    dot = warp_sum(dot) / H;
    float4* dxr = reinterpret_cast<float4*>(dx + g * sdx + (long long)r * H);
    uint2* d16 = dx16 ? reinterpret_cast<uint2*>(dx16 + g * sdx + (long long)r * H) : nullptr;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 a = wv[j], dd = d[j], xx = xv[j];
      const float4 xh = make_float4(xx.x * rs, xx.y * rs, xx.z * rs, xx.w * rs);
      float4 v = make_float4(rs * (a.x * dd.x - xh.x * dot), rs * (a.y * dd.y - xh.y * dot),
                             rs * (a.z * dd.z - xh.z * dot), rs * (a.w * dd.w - xh.w * dot));
      if (drr) {
        v.x += q[j].x;
        v.y += q[j].y;
        v.z += q[j].z;
        v.w += q[j].w;
      }
      dxr[lane + 32 * j] = v;
      if (d16) d16[lane + 32 * j] = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
      acc[j].x += dd.x * xh.x;
      acc[j].y += dd.y * xh.y;
      acc[j].z += dd.z * xh.z;
      acc[j].w += dd.w * xh.w;
    }
  }
  float4* mine = reinterpret_cast<float4*>(sdw + warp * H);
#pragma unroll
  for (int j = 0; j < NV; ++j) mine[lane + 32 * j] = acc[j];
  __syncthreads();
  float* out = dw_part + ((long long)g * nblk + b) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += sdw[k * H + i];
    out[i] = s;
  }
}

// dw[g][i] = sum_b dw_part[g][b][i] in a fixed order: eight interleaved running sums
// (block b feeds sum b % 8), so eight independent loads are in flight per thread instead
// of one dependent chain of nblk loads, then a fixed pairwise fold of the eight.
__global__ void reduce_parts_kernel(const float* __restrict__ part, int nblk, int H, int G, float* dw, long long sdw,
                                    float beta) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= G * H) return;
  const int g = idx / H, i = idx % H;
  const float* p = part + (long long)g * nblk * H + i;
  float s[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) s[k] = 0.f;
  int b = 0;
  for (; b + 8 <= nblk; b += 8) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = p[(long long)(b + k) * H];
#pragma unroll
    for (int k = 0; k < 8; ++k) s[k] += v[k];
  }
  for (int k = 0; b < nblk; ++b, ++k) s[k] += p[(long long)b * H];
  const float t = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
  float* d = dw + g * sdw + i;
  *d = beta != 0.f ? t + beta * *d : t;
}

// ids: [G][M] int32; E: group g's table at E + g*se ([V][H] fp32); out: [G][M][H] fp32.
__global__ void embedding_fwd_kernel(const int* __restrict__ ids, const float* __restrict__ E, long long se,
                                     float* __restrict__ out, int M, int H, int G, int V) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= G * M) return;
  const int g = warp / M;
  int id = ids[warp];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  const float4* src = reinterpret_cast<const float4*>(E + g * se + (long long)id * H);
  float4* dst = reinterpret_cast<float4*>(out + (long long)warp * H);
  for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
}

// One warp per token row. The row that first carries an id owns that id's gradient row.
__global__ void embedding_bwd_kernel(const int* __restrict__ ids, const float* __restrict__ dx, long long sdx,
                                     float* __restrict__ dE, long long se, int M, int H, int G, int V) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= G * M) return;
  const int g = warp / M, r = warp % M;
  const int* gid = ids + (long long)g * M;
  const int id = gid[r];
  // earlier occurrence? (warp-parallel scan of rows < r)
  bool dup = false;
  for (int j = lane; j < r; j += 32) dup |= (gid[j] == id);
  if (__any_sync(0xffffffffu, dup)) return;
  if (id < 0 || id >= V) return;
  // Gather every row carrying `id` (ballot over 32 rows at a time), summing in row order.
  const int nt = H / 32;
  float acc[64];
#pragma unroll
  for (int t = 0; t < 64; ++t) acc[t] = 0.f;
  for (int base = r; base < M; base += 32) {
    const int j = base + lane;
    unsigned m = __ballot_sync(0xffffffffu, j < M && gid[j] == id);
    while (m) {
      const int k = __ffs(m) - 1;
      m &= m - 1;
      const float* src = dx + g * sdx + (long long)(base + k) * H;
#pragma unroll
      for (int t = 0; t < 64; ++t)
        if (t < nt) acc[t] += src[t * 32 + lane];
    }
  }
  float* dst = dE + g * se + (long long)id * H;
#pragma unroll
  for (int t = 0; t < 64; ++t)
    if (t < nt) dst[t * 32 + lane] = acc[t];
}

// Deterministic O(M) embedding backward in two launches.
// 1. One CTA per path sorts the keys (token id << 12 | row) of its <= 4096 rows with a
//    bitonic network in shared memory, so every token's rows become one contiguous run
//    in increasing row order.
// 2. One warp per sorted position: the first position of each run sums the rows of the
//    run (row order, the same additions as embedding_bwd_kernel) into dE[id].
constexpr int kSortMax = 4096;

__global__ void __launch_bounds__(1024) embed_sort_kernel(const int* __restrict__ ids, int M,
                                                          unsigned* __restrict__ keys_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned k[kSortMax];
  const int g = blockIdx.x;
  int n = 1;
  while (n < M) n <<= 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    k[i] = i < M ? ((unsigned)ids[(long long)g * M + i] << 12) | (unsigned)i : 0xffffffffu;
  __syncthreads();
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned a = k[lo], b = k[hi];
        if ((a > b) == up) {
          k[lo] = b;
          k[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < M; i += blockDim.x) keys_out[(long long)g * M + i] = k[i];
}

template <int NT>
__global__ void embed_runs_kernel(const unsigned* __restrict__ keys, const float* __restrict__ dx, long long sdx,
                                  float* __restrict__ dE, long long se, int M, int H, int G, int V,
                                  uint8_t* __restrict__ rows, float* __restrict__ sq) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= G * M) return;
  const int g = warp / M, i = warp % M;
  const unsigned* gk = keys + (long long)g * M;
  const unsigned id = gk[i] >> 12;
  if (id >= (unsigned)V || (i > 0 && (gk[i - 1] >> 12) == id)) {
    if (sq && lane == 0) sq[(long long)g * M + i] = 0.f;  // not the start of a run
    return;
  }
  if (rows && lane == 0) rows[(long long)g * V + id] = 1;  // this row of dE is written below
  // end of this token's run: first sorted position whose id differs (32 keys per probe)
  int end = i + 1;
  while (true) {
    const int j = end + lane;
    const unsigned differ = __ballot_sync(0xffffffffu, j >= M || (gk[j] >> 12) != id);
    if (differ) {
      end += __ffs(differ) - 1;
      break;
    }
    end += 32;
  }
  const int nt = H / 32;
  constexpr int BATCH = NT <= 16 ? 8 : 2;  // rows loaded before they are added (in row order)
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  for (int j = i; j < end; j += BATCH) {
    float v[BATCH][NT];
#pragma unroll
    for (int b = 0; b < BATCH; ++b) {
      const bool in = j + b < end;
      const float* src = dx + g * sdx + (long long)(in ? (gk[j + b] & 0xfffu) : 0) * H;
#pragma unroll
      for (int t = 0; t < NT; ++t) v[b][t] = (in && t < nt) ? src[t * 32 + lane] : 0.f;
    }
#pragma unroll
    for (int b = 0; b < BATCH; ++b)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] += v[b][t];
  }
  float* dst = dE + g * se + (long long)id * H;
  float q = 0.f;
#pragma unroll
  for (int t = 0; t < NT; ++t)
    if (t < nt) {
      dst[t * 32 + lane] = acc[t];
      q = fmaf(acc[t], acc[t], q);
    }
  if (sq) {  // sum of squares of this gradient row, at the run's first sorted position
    q = warp_sum(q);
    if (lane == 0) sq[(long long)g * M + i] = q;
  }
}

}  // namespace odp

static inline int blocks_for(long long threads, int per) { return (int)((threads + per - 1) / per); }

// rows_per_warp: 1 or 4 forces the register-resident variant's rows per warp; 0 chooses
// four rows per warp, or one when four would leave fewer than two blocks per SM.
void rmsnorm_fwd_rpw(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor y, int64_t sy,
                     torch::Tensor rstd, int64_t M, int64_t H, int64_t G, double eps, int64_t rows_per_warp) {
  TORCH_CHECK(H % 128 == 0, "rmsnorm: hidden size must be a multiple of 128");
  TORCH_CHECK(rows_per_warp == 0 || rows_per_warp == 1 || rows_per_warp == 4, "rmsnorm: rows_per_warp is 0, 1 or 4");
  c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool reg = al16(x.data_ptr()) && al16(w.data_ptr()) && al16(y.data_ptr()) && sx % 4 == 0 && sw % 4 == 0 &&
                   sy % 4 == 0;
  const int nv = (int)(H / 128);
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const bool few = rows_per_warp ? rows_per_warp == 1 : G * M / 32 < 2 * sms;
#define ODP_RMS_FWD(NV)                                                                                          \
  if (reg && nv == NV) {                                                                                         \
    if (few)                                                                                                     \
      C10_CUDA_CHECK(odp::launch_pdl((odp::rmsnorm_fwd_reg_kernel<NV, 1>), dim3(blocks_for(G * M * 32, 256)), dim3(256), 0, st, \
          x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), sy,  \
          rstd.data_ptr<float>(), (int)M, (int)H, (int)G, (float)eps));                                           \
    else                                                                                                         \
      C10_CUDA_CHECK(odp::launch_pdl((odp::rmsnorm_fwd_reg_kernel<NV, 4>), dim3(blocks_for(G * M * 8, 256)), dim3(256), 0, st, \
          x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), sy,  \
          rstd.data_ptr<float>(), (int)M, (int)H, (int)G, (float)eps));                                           \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                              \
    return;                                                                                                      \
  }
  ODP_RMS_FWD(1) ODP_RMS_FWD(2) ODP_RMS_FWD(3) ODP_RMS_FWD(4) ODP_RMS_FWD(8)
#undef ODP_RMS_FWD
  C10_CUDA_CHECK(odp::launch_pdl((odp::rmsnorm_fwd_kernel), dim3(blocks_for(G * M * 32, 256)), dim3(256), 0, st, x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), sy,
      rstd.data_ptr<float>(), (int)M, (int)H, (int)G, (float)eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_fwd(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor y, int64_t sy,
                 torch::Tensor rstd, int64_t M, int64_t H, int64_t G, double eps) {
  rmsnorm_fwd_rpw(x, sx, w, sw, y, sy, rstd, M, H, G, eps, 0);
}

void rmsnorm_bwd(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor rstd, torch::Tensor dy,
                 int64_t sdy, c10::optional<torch::Tensor> dres, torch::Tensor dx, int64_t sdx,
                 c10::optional<torch::Tensor> dx16, torch::Tensor dw, int64_t sdw, torch::Tensor work, int64_t M,
                 int64_t H, int64_t G, double beta) {
  c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  // rows per block (32): 8-row blocks for few paths per GPU were measured slower (4x the
  // weight-gradient partials to write and reduce outweigh the extra parallelism)
  const int rpb = odp::kNormRowsPerBlock;
  const int nblk = (int)((M + rpb - 1) / rpb);
  TORCH_CHECK(work.numel() >= G * nblk * H, "rmsnorm_bwd: work buffer too small");
  auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  TORCH_CHECK(H % 4 == 0 && sx % 4 == 0 && sdy % 4 == 0 && sdx % 4 == 0 && sw % 4 == 0 && al16(x.data_ptr()) &&
                  al16(dy.data_ptr()) && al16(dx.data_ptr()) && al16(w.data_ptr()) &&
                  (!dres.has_value() || al16(dres->data_ptr())),
              "rmsnorm_bwd: rows are read as float4 (16-byte aligned bases, strides multiple of 4)");
  const size_t smem = 8 * H * sizeof(float);
  const int nv = (int)(H / 128);
  bool launched = false;
#define ODP_RMS_BWD(NV)                                                                                           \
  if (!launched && H % 128 == 0 && nv == NV) {                                                                    \
    if (smem > 48 * 1024)                                                                                         \
      cudaFuncSetAttribute(odp::rmsnorm_bwd_reg_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    C10_CUDA_CHECK(odp::launch_pdl((odp::rmsnorm_bwd_reg_kernel<NV>), dim3((int)G * nblk), dim3(256), smem, st, \
        x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, rstd.data_ptr<float>(), dy.data_ptr<float>(), sdy,      \
        dres.has_value() ? dres->data_ptr<float>() : nullptr, dx.data_ptr<float>(), sdx,                          \
        dx16.has_value() ? reinterpret_cast<__nv_bfloat16*>(dx16->data_ptr()) : nullptr, work.data_ptr<float>(),  \
        (int)M, (int)H, (int)G, rpb));                                                                             \
    launched = true;                                                                                              \
  }
  ODP_RMS_BWD(1) ODP_RMS_BWD(2) ODP_RMS_BWD(3) ODP_RMS_BWD(4) ODP_RMS_BWD(8)
#undef ODP_RMS_BWD
  if (!launched) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(odp::rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  C10_CUDA_CHECK(odp::launch_pdl((odp::rmsnorm_bwd_kernel), dim3((int)G * nblk), dim3(256), smem, st, x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, rstd.data_ptr<float>(), dy.data_ptr<float>(), sdy,
      dres.has_value() ? dres->data_ptr<float>() : nullptr, dx.data_ptr<float>(), sdx,
      dx16.has_value() ? reinterpret_cast<__nv_bfloat16*>(dx16->data_ptr()) : nullptr, work.data_ptr<float>(),
      (int)M, (int)H, (int)G, rpb));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  C10_CUDA_CHECK(odp::launch_pdl((odp::reduce_parts_kernel), dim3(blocks_for(G * H, 256)), dim3(256), 0, st, work.data_ptr<float>(), nblk, (int)H, (int)G,
                                                                    dw.data_ptr<float>(), sdw, (float)beta));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_fwd(torch::Tensor ids, torch::Tensor E, int64_t se, torch::Tensor out, int64_t M, int64_t H,
                   int64_t G, int64_t V) {
  TORCH_CHECK(H % 4 == 0, "embedding: hidden size must be a multiple of 4");
  c10::cuda::CUDAGuard guard(E.device());
  auto st = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(odp::launch_pdl((odp::embedding_fwd_kernel), dim3(blocks_for(G * M * 32, 256)), dim3(256), 0, st, ids.data_ptr<int>(), E.data_ptr<float>(), se, out.data_ptr<float>(), (int)M, (int)H, (int)G, (int)V));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_bwd(torch::Tensor ids, torch::Tensor dx, int64_t sdx, torch::Tensor dE, int64_t se, int64_t M,
                   int64_t H, int64_t G, int64_t V) {
  TORCH_CHECK(H % 32 == 0 && H <= 2048, "embedding_bwd: hidden size must be a multiple of 32 and <= 2048");
  c10::cuda::CUDAGuard guard(dE.device());
  auto st = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(odp::launch_pdl((odp::embedding_bwd_kernel), dim3(blocks_for(G * M * 32, 256)), dim3(256), 0, st, ids.data_ptr<int>(), dx.data_ptr<float>(), sdx, dE.data_ptr<float>(), se, (int)M, (int)H, (int)G, (int)V));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// embedding_bwd through a per-path sort (same result, O(M)); keys: [G][M] int32 scratch.
// Falls back to embedding_bwd for M > 4096 rows per path or V >= 2^20.
// sq (optional, fp32 [G][M]): sum of squares of each written gradient row at its run's
// first sorted position, 0 at the other positions (for the gradient-norm clip).
// rows (optional, uint8 [G][V]): cleared, then set to 1 for every vocabulary row whose
// gradient this call writes; the other rows of dE are left as they were (not zeroed), and
// consumers given `rows` read them as zero. Needs the sorted path (M <= 4096, V < 2^20).
void embedding_bwd_sorted(torch::Tensor ids, torch::Tensor dx, int64_t sdx, torch::Tensor dE, int64_t se, int64_t M,
                          int64_t H, int64_t G, int64_t V, torch::Tensor keys, c10::optional<torch::Tensor> rows,
                          c10::optional<torch::Tensor> sq) {
  if (M > odp::kSortMax || V >= (1 << 20)) {
    TORCH_CHECK(!rows.has_value() && !sq.has_value(),
                "embedding_bwd_sorted: touched-row flags and row sums of squares need M <= 4096 and V < 2^20");
    embedding_bwd(ids, dx, sdx, dE, se, M, H, G, V);
    return;
  }
  TORCH_CHECK(H % 32 == 0 && H <= 2048, "embedding_bwd: hidden size must be a multiple of 32 and <= 2048");
  TORCH_CHECK(keys.numel() >= G * M, "embedding_bwd_sorted: key scratch too small");
  c10::cuda::CUDAGuard guard(dE.device());
  auto st = at::cuda::getCurrentCUDAStream();
  unsigned* kp = reinterpret_cast<unsigned*>(keys.data_ptr<int>());
  uint8_t* rp = nullptr;
  if (rows.has_value()) {
    TORCH_CHECK(rows->numel() >= G * V && rows->scalar_type() == at::kByte, "embedding_bwd_sorted: rows is uint8 [G][V]");
    rp = rows->data_ptr<uint8_t>();
    C10_CUDA_CHECK(cudaMemsetAsync(rp, 0, (size_t)(G * V), st));
  }
  C10_CUDA_CHECK(odp::launch_pdl((odp::embed_sort_kernel), dim3((int)G), dim3(1024), 0, st, ids.data_ptr<int>(), (int)M, kp));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (H <= 512)
    C10_CUDA_CHECK(odp::launch_pdl((odp::embed_runs_kernel<16>), dim3(blocks_for(G * M * 32, 256)), dim3(256), 0, st, kp, dx.data_ptr<float>(), sdx, dE.data_ptr<float>(), se, (int)M, (int)H, (int)G, (int)V, rp,
        sq.has_value() ? sq->data_ptr<float>() : nullptr));
  else
    C10_CUDA_CHECK(odp::launch_pdl((odp::embed_runs_kernel<64>), dim3(blocks_for(G * M * 32, 256)), dim3(256), 0, st, kp, dx.data_ptr<float>(), sdx, dE.data_ptr<float>(), se, (int)M, (int)H, (int)G, (int)V, rp,
        sq.has_value() ? sq->data_ptr<float>() : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
