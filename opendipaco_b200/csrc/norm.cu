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

// dy: [G][M][H] fp32 (grad w.r.t. the norm output); dres: optional residual grad added to dx.
// dx may alias dres. dw_part: [G][nblk][H] partial sums of dy*xhat for rows of each block.
constexpr int kNormRowsPerBlock = 32;

__global__ void rmsnorm_bwd_kernel(const float* __restrict__ x, long long sx, const float* __restrict__ w,
                                   long long sw, const float* __restrict__ rstd, const float* __restrict__ dy,
                                   long long sdy, const float* dres, float* dx, long long sdx,
                                   __nv_bfloat16* dx16, float* __restrict__ dw_part, int M, int H, int G) {
  // block = 256 threads = 8 warps; block handles kNormRowsPerBlock rows of one group
  const int nblk = (M + kNormRowsPerBlock - 1) / kNormRowsPerBlock;
  const int g = blockIdx.x / nblk, b = blockIdx.x % nblk;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  extern __shared__ float sdw[];  // [8 warps][H]
  for (int i = threadIdx.x; i < 8 * H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  const float* wg = w + g * sw;
  for (int rr = warp; rr < kNormRowsPerBlock; rr += 8) {
    const int r = b * kNormRowsPerBlock + rr;
    if (r >= M) break;
    const float* xr = x + g * sx + (long long)r * H;
    const float* dyr = dy + g * sdy + (long long)r * H;
    const float rs = rstd[(long long)g * M + r];
    float dot = 0.f;
    for (int i = lane; i < H; i += 32) dot += wg[i] * dyr[i] * (xr[i] * rs);
    dot = warp_sum(dot) / H;
    float* dxr = dx + g * sdx + (long long)r * H;
    const float* drr = dres ? dres + g * sdx + (long long)r * H : nullptr;
    for (int i = lane; i < H; i += 32) {
      const float xh = xr[i] * rs;
      float v = rs * (wg[i] * dyr[i] - xh * dot);
      if (drr) v += drr[i];
      dxr[i] = v;
      if (dx16) dx16[g * sdx + (long long)r * H + i] = __float2bfloat16(v);
      sdw[warp * H + i] += dyr[i] * xh;
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

// dw[g][i] = sum_b dw_part[g][b][i] in fixed order.
__global__ void reduce_parts_kernel(const float* __restrict__ part, int nblk, int H, int G, float* dw, long long sdw,
                                    float beta) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= G * H) return;
  const int g = idx / H, i = idx % H;
  const float* p = part + (long long)g * nblk * H + i;
  float s = 0.f;
  for (int b = 0; b < nblk; ++b) s += p[(long long)b * H];
  float* d = dw + g * sdw + i;
  *d = beta != 0.f ? s + beta * *d : s;
}

// ids: [G][M] int32; E: group g's table at E + g*se ([V][H] fp32); out: [G][M][H] fp32.
__global__ void embedding_fwd_kernel(const int* __restrict__ ids, const float* __restrict__ E, long long se,
                                     float* __restrict__ out, int M, int H, int G, int V) {
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

}  // namespace odp

static inline int blocks_for(long long threads, int per) { return (int)((threads + per - 1) / per); }

void rmsnorm_fwd(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor y, int64_t sy,
                 torch::Tensor rstd, int64_t M, int64_t H, int64_t G, double eps) {
  TORCH_CHECK(H % 128 == 0, "rmsnorm: hidden size must be a multiple of 128");
  c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  odp::rmsnorm_fwd_kernel<<<blocks_for(G * M * 32, 256), 256, 0, st>>>(
      x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), sy,
      rstd.data_ptr<float>(), (int)M, (int)H, (int)G, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor rstd, torch::Tensor dy,
                 int64_t sdy, c10::optional<torch::Tensor> dres, torch::Tensor dx, int64_t sdx,
                 c10::optional<torch::Tensor> dx16, torch::Tensor dw, int64_t sdw, torch::Tensor work, int64_t M,
                 int64_t H, int64_t G, double beta) {
  c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int nblk = (int)((M + odp::kNormRowsPerBlock - 1) / odp::kNormRowsPerBlock);
  TORCH_CHECK(work.numel() >= G * nblk * H, "rmsnorm_bwd: work buffer too small");
  const size_t smem = 8 * H * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(odp::rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  odp::rmsnorm_bwd_kernel<<<(int)G * nblk, 256, smem, st>>>(
      x.data_ptr<float>(), sx, w.data_ptr<float>(), sw, rstd.data_ptr<float>(), dy.data_ptr<float>(), sdy,
      dres.has_value() ? dres->data_ptr<float>() : nullptr, dx.data_ptr<float>(), sdx,
      dx16.has_value() ? reinterpret_cast<__nv_bfloat16*>(dx16->data_ptr()) : nullptr, work.data_ptr<float>(),
      (int)M, (int)H, (int)G);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  odp::reduce_parts_kernel<<<blocks_for(G * H, 256), 256, 0, st>>>(work.data_ptr<float>(), nblk, (int)H, (int)G,
                                                                    dw.data_ptr<float>(), sdw, (float)beta);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_fwd(torch::Tensor ids, torch::Tensor E, int64_t se, torch::Tensor out, int64_t M, int64_t H,
                   int64_t G, int64_t V) {
  TORCH_CHECK(H % 4 == 0, "embedding: hidden size must be a multiple of 4");
  c10::cuda::CUDAGuard guard(E.device());
  auto st = at::cuda::getCurrentCUDAStream();
  odp::embedding_fwd_kernel<<<blocks_for(G * M * 32, 256), 256, 0, st>>>(
      ids.data_ptr<int>(), E.data_ptr<float>(), se, out.data_ptr<float>(), (int)M, (int)H, (int)G, (int)V);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_bwd(torch::Tensor ids, torch::Tensor dx, int64_t sdx, torch::Tensor dE, int64_t se, int64_t M,
                   int64_t H, int64_t G, int64_t V) {
  TORCH_CHECK(H % 32 == 0 && H <= 2048, "embedding_bwd: hidden size must be a multiple of 32 and <= 2048");
  c10::cuda::CUDAGuard guard(dE.device());
  auto st = at::cuda::getCurrentCUDAStream();
  odp::embedding_bwd_kernel<<<blocks_for(G * M * 32, 256), 256, 0, st>>>(
      ids.data_ptr<int>(), dx.data_ptr<float>(), sdx, dE.data_ptr<float>(), se, (int)M, (int)H, (int)G, (int)V);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
