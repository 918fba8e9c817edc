// Routing kernels.
//
// bag_of_tokens: features of a token prefix = L2-normalise(mean of the projection
//   rows of its tokens) (== normalised counts @ projection). One CTA per prefix,
//   threads over feature columns, fixed summation order (deterministic).
//
// kmeans_assign_tc: the k-means assignment as a tensor-core contraction. A CTA takes
//   128 points (one TMEM lane each) against a block of up to 256 centroids (TMEM
//   columns) and computes x.c with tcgen05.mma kind::tf32 in three products, the
//   "3xTF32" split of Ootomo and Yokota (2022): with hi(v) = v with its low 13 mantissa
//   bits cleared (exact in tf32) and lo(v) = v - hi(v) (exact in fp32),
//     x.c ~= hi(x).hi(c) + hi(x).lo(c) + lo(x).hi(c),
//   accumulated in fp32 in TMEM, which keeps the dot product to about 1e-6 relative to
//   |x||c| -- fp32 quality, so assignments agree with an fp32 cdist except on
//   near-ties. Operands are staged from global memory by plain 16-byte loads (one point
//   row per thread: 128 contiguous bytes per 32-feature chunk) into 128-byte-swizzled
//   K-major tiles, double-buffered so the next chunk's staging overlaps the MMAs.
//   The epilogue is one thread per point: it reads its TMEM row, forms
//   |x|^2 - 2 x.c + |c|^2 (norms summed in fixed order while staging) and keeps the k
//   nearest (k <= 8) by insertion (ties: lower index first), carried across centroid
//   blocks, so any number of centroids works.
//
// kmeans_partial_sums: the centroid update without float atomics. Grid (K, S): CTA
//   (k, s) walks its contiguous slice of the points in order, compacts the indices
//   assigned to k (warp ballots, block prefix) and adds their rows in index order, one
//   feature column per thread. The S partials are then summed in a fixed order, so the
//   fit is bitwise reproducible.
//
// Reference: the assignment and update loop of src/opendipaco/routing/kmeans.py:20-55
// (torch.cdist + argmin, per-cluster masked means).
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

namespace km {

constexpr int T = 128;           // points per CTA (TMEM lanes)
constexpr int KB = 256;          // centroids per block (TMEM columns, UMMA N <= 256)
constexpr int CH = 32;           // features per chunk: one 128-byte swizzled row of fp32
constexpr int ATILE = T * 128;   // bytes of one 128 x 32 fp32 tile

// Instruction descriptor, kind::tf32: D = f32, A = B = tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

ODP_DEVICE void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}

// Byte offset of the 16-byte chunk j (4 fp32) of row r in a 128-byte-swizzled tile.
ODP_DEVICE uint32_t swz(int r, int j) { return (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4)); }

// K-major descriptor of a swizzled tile, k-step kk = 8 tf32 = 32 bytes.
ODP_DEVICE uint64_t desc(uint32_t tile, int kk) { return umma_smem_desc(tile + kk * 32, 16, 1024, kLayoutSW128); }

ODP_DEVICE float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// Split one 32-feature chunk of a row into its hi / lo tiles; returns the chunk's sum
// of squares (fixed order). Rows past `n` are zero.
ODP_DEVICE float stage_row(uint8_t* hi, uint8_t* lo, const float* __restrict__ src, int D, int row, int r,
                           int n, int c0) {
  float ss = 0.f;
  const bool live = r < n;
  const float4* p = reinterpret_cast<const float4*>(src + (long long)r * D + c0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 v = live ? __ldg(p + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v.x * v.x;
    ss += v.y * v.y;
    ss += v.z * v.z;
    ss += v.w * v.w;
    const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
    const float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    *reinterpret_cast<float4*>(hi + swz(row, j)) = h;
    *reinterpret_cast<float4*>(lo + swz(row, j)) = l;
  }
  return ss;
}

struct Smem {
  uint64_t bar[2];
  uint32_t tmem;
  float cn[KB];
};

}  // namespace km

// One CTA: points [128 b, 128 b + 128) against all K centroids, in blocks of up to 256.
// smem per buffer: A hi / lo (2 x 16 KB) + B hi / lo (2 x kb x 128 B); two buffers.
__global__ void __launch_bounds__(128) kmeans_assign_tc_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ c, int N, int K, int D,
                                                               int topk, int kb_max, long long* __restrict__ idx_out,
                                                               float* __restrict__ mind_out,
                                                               float* __restrict__ dist_out, int* err) {
  using namespace km;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int btile = kb_max * 128;
  const int buf_bytes = 2 * ATILE + 2 * btile;
  __shared__ Smem s;
  const int tid = threadIdx.x, warp = tid / 32;
  const int p0 = blockIdx.x * T;
  uint32_t ncols = 32;
  while ((int)ncols < kb_max) ncols <<= 1;
  if (tid == 0) {
    mbar_init(&s.bar[0], 1);
    mbar_init(&s.bar[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&s.tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;

  float best_d[8];
  int best_i[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    best_d[j] = INFINITY;
    best_i[j] = 0x7fffffff;
  }
  float xn = 0.f;
  uint32_t phase[2] = {0u, 0u};
  bool ok = true;
  const int nch = D / CH;

  for (int k0 = 0; k0 < K && ok; k0 += kb_max) {
    const int kb = min(kb_max, K - k0);
    const int kbp = (kb + 15) & ~15;  // UMMA N: a multiple of 16 (padded centroids are zero)
    const uint32_t idesc = idesc_tf32(T, kbp);
    float cn0 = 0.f, cn1 = 0.f, xs = 0.f;
    auto stage = [&](int ch, int b) {
      uint8_t* base = sm + b * buf_bytes;
      uint8_t *ah = base, *al = base + ATILE, *bh = base + 2 * ATILE, *bl = bh + btile;
      xs += stage_row(ah, al, x, D, tid, p0 + tid, N, ch * CH);
      if (tid < kbp) cn0 += stage_row(bh, bl, c, D, tid, k0 + tid, k0 + kb, ch * CH);
      if (tid + T < kbp) cn1 += stage_row(bh, bl, c, D, tid + T, k0 + tid + T, k0 + kb, ch * CH);
    };
    stage(0, 0);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    for (int ch = 0; ch < nch && ok; ++ch) {
      const int b = ch & 1;
      if (tid == 0) {
        const uint32_t base = smem_u32(sm + b * buf_bytes);
        const uint32_t ah = base, al = base + ATILE, bh = base + 2 * ATILE, bl = bh + btile;
#pragma unroll
        for (int kk = 0; kk < CH / 8; ++kk) {
          const uint32_t acc0 = (ch | kk) ? 1u : 0u;
          umma_tf32(tmem, desc(ah, kk), desc(bh, kk), idesc, acc0);
          umma_tf32(tmem, desc(ah, kk), desc(bl, kk), idesc, 1u);
          umma_tf32(tmem, desc(al, kk), desc(bh, kk), idesc, 1u);
        }
        umma_commit(&s.bar[b]);
      }
      if (ch + 1 < nch) {
        if (ch >= 1) {  // the MMAs of chunk ch - 1 read the buffer about to be refilled
          if (tid == 0) ok = mbar_wait(&s.bar[b ^ 1], phase[b ^ 1], err, ERR_TIMEOUT_ACCUM);
          phase[b ^ 1] ^= 1u;
          ok = __syncthreads_and(ok);
          tc_fence_after();
          if (!ok) break;
        }
        stage(ch + 1, b ^ 1);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
      }
    }
    // Drain: wait for the commits not waited above (chunks nch - 2 and nch - 1).
    for (int ch = (nch >= 2 ? nch - 2 : 0); ch < nch; ++ch) {
      const int b = ch & 1;
      if (ok && tid == 0) ok = mbar_wait(&s.bar[b], phase[b], err, ERR_TIMEOUT_ACCUM);
      phase[b] ^= 1u;
    }
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (tid < kbp) s.cn[tid] = cn0;
    if (tid + T < kbp) s.cn[tid + T] = cn1;
    xn = xs;
    __syncthreads();
    if (!ok) break;

    // Epilogue: this thread's point against the block's centroids.
    const int p = p0 + tid;
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    for (int col = 0; col < kbp; col += 16) {
      float dot[16];
      tmem_ld16(lane_addr + col, dot);
      if (p >= N) continue;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int kl = col + e;
        if (kl >= kb) break;
        const int k = k0 + kl;
        const float dist = xn - 2.f * dot[e] + s.cn[kl];
        if (dist_out) dist_out[(long long)p * K + k] = dist;
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
    }
    // TMEM and the staging buffers are reused by the next block.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  const int p = p0 + tid;
  if (p < N) {
    for (int j = 0; j < topk; ++j) idx_out[(long long)p * topk + j] = best_i[j];
    if (mind_out) mind_out[p] = best_d[0];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// CTA (k, s): sum of the rows of points [s * per, (s + 1) * per) assigned to cluster k,
// in index order; one feature column per thread (D <= 4 * blockDim).
__global__ void __launch_bounds__(256) kmeans_partial_sums_kernel(const float* __restrict__ x, int D,
                                                                  const long long* __restrict__ assign,
                                                                  int stride, int N, int per, int K,
                                                                  float* __restrict__ sums,
                                                                  int* __restrict__ counts) {
  const int k = blockIdx.x, sl = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int list[256];
  __shared__ int wtot[8];
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int count = 0;
  const int a = sl * per, b = min(N, a + per);
  for (int base = a; base < b; base += 256) {
    const int i = base + tid;
    const bool hit = i < b && assign[(long long)i * stride] == k;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) wtot[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      before += w < warp ? wtot[w] : 0;
      total += wtot[w];
    }
    if (hit) list[before + __popc(m & ((1u << lane) - 1u))] = i;
    __syncthreads();
    for (int j = 0; j < total; ++j) {
      const float* row = x + (long long)list[j] * D;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int f = tid + q * 256;
        if (f < D) acc[q] += row[f];
      }
    }
    count += total;
    __syncthreads();
  }
  float* out = sums + ((long long)sl * K + k) * D;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int f = tid + q * 256;
    if (f < D) out[f] = acc[q];
  }
  if (tid == 0) counts[sl * K + k] = count;
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

// [N, topk] nearest centroids, plus (optionally) the [N] nearest squared distance and the
// [N, K] squared distances. x and c are fp32 with rows of D features, D a multiple of 32
// (callers pad with zeros, which changes no distance).
std::vector<torch::Tensor> kmeans_assign(torch::Tensor x, torch::Tensor c, int64_t topk, bool want_min,
                                         bool want_dist, torch::Tensor err) {
  TORCH_CHECK(topk >= 1 && topk <= 8, "kmeans_assign: topk in [1, 8]");
  TORCH_CHECK(x.is_cuda() && c.is_cuda() && x.scalar_type() == torch::kFloat && c.scalar_type() == torch::kFloat,
              "kmeans_assign: fp32 CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && c.dim() == 2 && x.size(1) == c.size(1), "kmeans_assign: x [N, D], c [K, D]");
  TORCH_CHECK(x.is_contiguous() && c.is_contiguous(), "kmeans_assign: contiguous rows");
  const int N = (int)x.size(0), D = (int)x.size(1), K = (int)c.size(0);
  TORCH_CHECK(D % 32 == 0 && D > 0, "kmeans_assign: feature dim must be a positive multiple of 32");
  TORCH_CHECK(K >= 1 && topk <= K, "kmeans_assign: need topk <= K");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0,
              "kmeans_assign: 16-byte aligned rows");
  c10::cuda::CUDAGuard guard(x.device());
  auto idx = torch::empty({N, topk}, x.options().dtype(torch::kLong));
  auto mind = want_min ? torch::empty({N}, x.options()) : torch::Tensor();
  auto dist = want_dist ? torch::empty({N, K}, x.options()) : torch::Tensor();
  if (N == 0) return {idx, mind, dist};
  const int kb_max = std::min(K, odp::km::KB);
  const int kbp = (kb_max + 15) & ~15;
  const int smem = 2 * (2 * odp::km::ATILE + 2 * kbp * 128) + 1024;
  auto kern = odp::kmeans_assign_tc_kernel;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kern<<<(N + odp::km::T - 1) / odp::km::T, odp::km::T, smem, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), c.data_ptr<float>(), N, K, D, (int)topk, kbp,
      reinterpret_cast<long long*>(idx.data_ptr<int64_t>()), want_min ? mind.data_ptr<float>() : nullptr,
      want_dist ? dist.data_ptr<float>() : nullptr, err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {idx, mind, dist};
}

// Per-cluster sums and counts of the points whose first assignment column is the
// cluster: ([K, D] fp32 sums, [K] int32 counts), reproducible bit for bit.
std::vector<torch::Tensor> kmeans_cluster_sums(torch::Tensor x, torch::Tensor assign, int64_t K) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous() && x.dim() == 2,
              "kmeans_cluster_sums: x fp32 [N, D] contiguous");
  TORCH_CHECK(assign.is_cuda() && assign.scalar_type() == torch::kLong && assign.dim() == 2 &&
                  assign.size(0) == x.size(0) && assign.is_contiguous(),
              "kmeans_cluster_sums: assign int64 [N, k]");
  const int N = (int)x.size(0), D = (int)x.size(1);
  TORCH_CHECK(D <= 1024, "kmeans_cluster_sums: feature dim <= 1024");
  c10::cuda::CUDAGuard guard(x.device());
  const int S = std::max(1, std::min(64, (N + 2047) / 2048));
  const int per = (N + S - 1) / S;
  auto part = torch::empty({S, K, D}, x.options());
  auto cnt = torch::empty({S, K}, x.options().dtype(torch::kInt));
  if (N > 0)
    odp::kmeans_partial_sums_kernel<<<dim3((unsigned)K, (unsigned)S), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        x.data_ptr<float>(), D, reinterpret_cast<const long long*>(assign.data_ptr<int64_t>()),
        (int)assign.size(1), N, per, (int)K, part.data_ptr<float>(), cnt.data_ptr<int>());
  else {
    part.zero_();
    cnt.zero_();
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  // Fixed-order reduction over the S slices (the partials are summed in slice order).
  auto sums = part.select(0, 0).clone();
  for (int s = 1; s < S; ++s) sums.add_(part.select(0, s));
  return {sums, at::sum(cnt, {0}, false, at::kInt)};
}
