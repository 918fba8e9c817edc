// Routing kernels.
//
// bag_of_tokens: features of a token prefix = L2-normalise(mean of the projection
//   rows of its tokens) (== normalised counts @ projection). One CTA per prefix,
//   threads over feature columns, fixed summation order (deterministic).
// kmeans_assign: squared distances |x|^2 - 2 x.c + |c|^2 of every point to every
//   centroid (K <= 64), one warp per point, and the k nearest (k <= 8) by an
//   in-register insertion, ties broken by the lower index. Optionally also writes the
//   [N, K] distance matrix (used by the centroid update of the k-means fit).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

__global__ void bag_of_tokens_kernel(const int* __restrict__ ids, const long long* __restrict__ offs,
                                     const float* __restrict__ proj, int F, int V, float* __restrict__ out) {
  const int i = blockIdx.x;
  const long long a = offs[i], b = offs[i + 1];
  __shared__ float red[32];
  float local[8];
  int nloc = 0;
  float ss = 0.f;
  for (int f = threadIdx.x; f < F; f += blockDim.x) {
    float s = 0.f;
    for (long long t = a; t < b; ++t) {
      int id = ids[t];
      id = id < 0 ? 0 : (id >= V ? V - 1 : id);
      s += proj[(long long)id * F + f];
    }
    s = b > a ? s / (float)(b - a) : 0.f;
    local[nloc++] = s;
    ss += s * s;
  }
  ss = warp_sum(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < (int)blockDim.x / 32; ++k) t += red[k];
    red[0] = t;
  }
  __syncthreads();
  const float nrm = fmaxf(sqrtf(red[0]), 1e-12f);
  nloc = 0;
  for (int f = threadIdx.x; f < F; f += blockDim.x) out[(long long)i * F + f] = local[nloc++] / nrm;
}

__global__ void kmeans_assign_kernel(const float* __restrict__ x, const float* __restrict__ c,
                                     const float* __restrict__ cn, int N, int K, int D, int topk,
                                     long long* __restrict__ idx_out, float* __restrict__ dist_out) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (w >= N) return;
  const float* xr = x + (long long)w * D;
  float xn = 0.f;
  for (int d = lane; d < D; d += 32) xn += xr[d] * xr[d];
  xn = warp_sum(xn);
  float best_d[8];
  int best_i[8];
  for (int j = 0; j < 8; ++j) {
    best_d[j] = INFINITY;
    best_i[j] = 0x7fffffff;
  }
  for (int k = 0; k < K; ++k) {
    const float* cr = c + (long long)k * D;
    float dot = 0.f;
    for (int d = lane; d < D; d += 32) dot += xr[d] * cr[d];
    dot = warp_sum(dot);
    const float dist = xn - 2.f * dot + cn[k];
    if (dist_out && lane == 0) dist_out[(long long)w * K + k] = dist;
    // insertion into the sorted top-k (all lanes hold identical copies)
    if (dist < best_d[topk - 1]) {
      int j = topk - 1;
      while (j > 0 && best_d[j - 1] > dist) {
        best_d[j] = best_d[j - 1];
        best_i[j] = best_i[j - 1];
        --j;
      }
      best_d[j] = dist;
      best_i[j] = k;
    }
  }
  if (lane == 0)
    for (int j = 0; j < topk; ++j) idx_out[(long long)w * topk + j] = best_i[j];
}

}  // namespace odp

torch::Tensor bag_of_tokens(torch::Tensor ids, torch::Tensor offs, torch::Tensor proj) {
  c10::cuda::CUDAGuard guard(proj.device());
  const int N = (int)offs.numel() - 1, V = (int)proj.size(0), F = (int)proj.size(1);
  TORCH_CHECK(F <= 256 * 8, "bag_of_tokens: feature_dim too large");
  auto out = torch::empty({N, F}, proj.options());
  if (N > 0)
    odp::bag_of_tokens_kernel<<<N, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        ids.data_ptr<int>(), reinterpret_cast<const long long*>(offs.data_ptr<int64_t>()), proj.data_ptr<float>(),
        F, V, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

std::vector<torch::Tensor> kmeans_assign(torch::Tensor x, torch::Tensor c, int64_t topk, bool want_dist) {
  TORCH_CHECK(topk >= 1 && topk <= 8, "kmeans_assign: topk in [1, 8]");
  c10::cuda::CUDAGuard guard(x.device());
  auto xf = x.to(torch::kFloat).contiguous(), cf = c.to(torch::kFloat).contiguous();
  const int N = (int)xf.size(0), D = (int)xf.size(1), K = (int)cf.size(0);
  auto cn = (cf * cf).sum(1).contiguous();
  auto idx = torch::empty({N, topk}, x.options().dtype(torch::kLong));
  auto dist = want_dist ? torch::empty({N, K}, xf.options()) : torch::Tensor();
  if (N > 0)
    odp::kmeans_assign_kernel<<<(N * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        xf.data_ptr<float>(), cf.data_ptr<float>(), cn.data_ptr<float>(), N, K, D, (int)topk,
        reinterpret_cast<long long*>(idx.data_ptr<int64_t>()), want_dist ? dist.data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {idx, dist};
}
