// Cross-entropy over bf16 logits produced by the LM-head GEMM.
//
// The LM-head GEMM epilogue already wrote, for every row and every 128-column vocab
// tile, the (max, sum exp) of the bf16-rounded logits. ce_finalize merges those
// partials into the row log-sum-exp and the per-row loss lse - logit[target]
// (ignore_index -100), then a fixed-order block reduction gives each path's loss sum
// and valid-token count. ce_backward overwrites the logits in place with
// dlogits = (softmax - onehot) / count (bf16), which the two backward GEMMs consume.
//
// ce_fused does loss and dlogits in one pass when the GEMM wrote plain bf16 logits: one
// CTA per row keeps the row in registers, so the logits are read once and written once.
//
// cross_entropy_rows computes the same per-row loss straight from a logits tensor
// (eval / EM scoring), one CTA per row.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

// Per-row arrays (labels, lse, row_loss) of group g start at g * ms (ms = M unless the
// call covers a chunk of each group's rows, the pointers then offset to the chunk).
__global__ void ce_finalize_kernel(const float2* __restrict__ part, int T, const __nv_bfloat16* __restrict__ logits,
                                   long long ldl, long long sl, const int* __restrict__ labels, int M, int G,
                                   float* __restrict__ lse, float* __restrict__ row_loss, long long ms) {
  pdl_wait();
  pdl_trigger();
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= G * M) return;
  const long long r = (long long)(q / M) * ms + q % M;
  const float2* p = part + (long long)q * T;
  float mx = -INFINITY;
  for (int t = 0; t < T; ++t) mx = fmaxf(mx, p[t].x);
  float s = 0.f;
  for (int t = 0; t < T; ++t) s += p[t].y * __expf(p[t].x - mx);
  const float l = mx + logf(s);
  lse[r] = l;
  const int y = labels[r];
  const int g = q / M, m = q % M;
  float loss = 0.f;
  if (y >= 0) loss = l - __bfloat162float(logits[g * sl + (long long)m * ldl + y]);
  row_loss[r] = loss;
}

// One block per group: loss_sum[g] = sum of row losses (fixed order), count[g] = valid rows.
// With inv_given (the normaliser of a batch split over several GPUs, known on the host)
// the mean uses it and out_inv_count is left alone.
__global__ void group_sum_kernel(const float* __restrict__ row_loss, const int* __restrict__ labels, int M,
                                 float* __restrict__ out_sum, float* __restrict__ out_inv_count,
                                 float* __restrict__ out_loss, const float* __restrict__ inv_given) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x;
  __shared__ float ss[256];
  __shared__ int sc[256];
  float s = 0.f;
  int c = 0;
  for (int i = threadIdx.x; i < M; i += blockDim.x) {
    s += row_loss[(long long)g * M + i];
    c += labels[(long long)g * M + i] >= 0;
  }
  ss[threadIdx.x] = s;
  sc[threadIdx.x] = c;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      ss[threadIdx.x] += ss[threadIdx.x + o];
      sc[threadIdx.x] += sc[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out_sum[g] = ss[0];
    if (inv_given) {
      if (out_loss) out_loss[g] = ss[0] * inv_given[g];
    } else {
      const float cnt = (float)(sc[0] > 0 ? sc[0] : 1);
      out_inv_count[g] = 1.f / cnt;
      if (out_loss) out_loss[g] = ss[0] / cnt;
    }
  }
}

// In place: logits -> (softmax - onehot) * inv_count[g]; 8 bf16 per thread.
__global__ void ce_backward_kernel(__nv_bfloat16* logits, long long ldl, long long sl, const float* __restrict__ lse,
                                   const int* __restrict__ labels, const float* __restrict__ inv_count, int M, int V,
                                   int G, long long ms) {
  pdl_wait();
  pdl_trigger();
  const long long vec_per_row = V / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)G * M * vec_per_row) return;
  const long long q = idx / vec_per_row;
  const int c0 = (int)(idx % vec_per_row) * 8;
  const int g = (int)(q / M), m = (int)(q % M);
  const long long r = (long long)g * ms + m;
  uint4* ptr = reinterpret_cast<uint4*>(logits + g * sl + (long long)m * ldl + c0);
  const int y = labels[r];
  if (y < 0) {
    *ptr = make_uint4(0, 0, 0, 0);
    return;
  }
  const float l = lse[r], sc = inv_count[g];
  uint4 v = *ptr;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&v);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    float p0 = __expf(__bfloat162float(x[e]) - l), p1 = __expf(__bfloat162float(x[e + 1]) - l);
    if (c0 + e == y) p0 -= 1.f;
    if (c0 + e + 1 == y) p1 -= 1.f;
    o[e / 2] = pack_bf16(p0 * sc, p1 * sc);
  }
  *ptr = make_uint4(o[0], o[1], o[2], o[3]);
}

// inv_count[g] = 1 / max(1, #labels >= 0 of group g): the dlogits scale, known before the loss.
__global__ void label_count_kernel(const int* __restrict__ labels, int M, float* __restrict__ inv_count) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x;
  __shared__ int sc[256];
  int c = 0;
  for (int i = threadIdx.x; i < M; i += blockDim.x) c += labels[(long long)g * M + i] >= 0;
  sc[threadIdx.x] = c;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) sc[threadIdx.x] += sc[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) inv_count[g] = 1.f / (float)(sc[0] > 0 ? sc[0] : 1);
}

constexpr int kCeThreads = 256;
constexpr int kCeMaxV = 32768;  // the row (<= 64 KB of bf16) is staged in shared memory

constexpr float kLog2e = 1.4426950408889634f;

// Two packed bf16 maxima (max.bf16x2) and the hardware base-2 exponential (ex2.approx).
ODP_DEVICE uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
ODP_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
ODP_DEVICE float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
ODP_DEVICE float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// One CTA per row. The whole bf16 row is brought into shared memory with one bulk copy
// (completion on an mbarrier, bounded wait), then
//   max (packed bf16 pairs), sum exp -> lse = max + log(sum),  loss = lse - x[label]
//   dlogits = (exp(x - lse) - onehot(label)) * inv_count[g]   written in place as bf16.
// Rows with label < 0 get loss 0 and zero dlogits. 64 KB per CTA: three CTAs per SM
// overlap one row's copy with another's arithmetic.
// GRAD = false (ce_stats): passes 1 and 2 only -- the logits are read, not rewritten -- and
// ob = ce_ob(lse, sc) is written per row for the LM-head gradient GEMMs, which form the
// same dlogits from the logits while staging their operand.
template <bool GRAD>
__global__ void __launch_bounds__(kCeThreads) ce_fused_kernel(__nv_bfloat16* logits, long long ldl, long long sl,
                                                              const int* __restrict__ labels, int M, int V,
                                                              const float* __restrict__ inv_count,
                                                              float* __restrict__ lse_out, float* __restrict__ row_loss,
                                                              int* err, long long ms, float* __restrict__ ob_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t ce_smem[];
  __shared__ uint64_t bar;
  __shared__ float red_m[kCeThreads / 32], red_s[kCeThreads / 32];
  const int g = (int)(blockIdx.x / M), m = (int)(blockIdx.x % M);
  const long long r = (long long)g * ms + m;  // index of the per-row arrays
  __nv_bfloat16* rowp = logits + g * sl + (long long)m * ldl;
  uint4* row = reinterpret_cast<uint4*>(rowp);
  const int nvec = V / 8;
  const int y = labels[r];
  if (y < 0) {
    if (GRAD)
      for (int i = threadIdx.x; i < nvec; i += kCeThreads) row[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
      row_loss[r] = 0.f;
      lse_out[r] = 0.f;
      if (!GRAD) ob_out[r] = 0.f;
    }
    return;
  }
  const uint4* srow = reinterpret_cast<const uint4*>(ce_smem);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t bytes = (uint32_t)V * 2;
    mbar_expect_tx(&bar, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(ce_smem)),
                 "l"(rowp), "r"(bytes), "r"(smem_u32(&bar))
                 : "memory");
  }
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0, err, ERR_TIMEOUT_FULL);
  // pass 1: row max on packed bf16 pairs (exact in bf16)
  uint32_t m2 = 0xff80ff80u;  // (-inf, -inf)
  if (ok) {
    for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
      const uint4 v = srow[i];
      m2 = bmax2(m2, bmax2(bmax2(v.x, v.y), bmax2(v.z, v.w)));
    }
  }
  float mx = fmaxf(bf_lo(m2), bf_hi(m2));
  mx = warp_max(mx);
  if (threadIdx.x % 32 == 0) red_m[threadIdx.x / 32] = mx;
  __syncthreads();
  mx = red_m[0];
#pragma unroll
  for (int w = 1; w < kCeThreads / 32; ++w) mx = fmaxf(mx, red_m[w]);
  // pass 2: sum of exp(x - max) as 2^(x log2e - max log2e)
  const float mb = mx * kLog2e;
  float se0 = 0.f, se1 = 0.f;
  if (ok) {
    for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
      const uint4 v = srow[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        se0 += ex2_approx(fmaf(bf_lo(w[e]), kLog2e, -mb));
        se1 += ex2_approx(fmaf(bf_hi(w[e]), kLog2e, -mb));
      }
    }
  }
  float se = warp_sum(se0 + se1);
  if (threadIdx.x % 32 == 0) red_s[threadIdx.x / 32] = se;
  __syncthreads();
  se = 0.f;
#pragma unroll
  for (int w = 0; w < kCeThreads / 32; ++w) se += red_s[w];
  if (!ok) return;  // the error word tells the host; this row is left as it was
  const float l = mx + logf(se);
  const float sc = inv_count[g];
  if (threadIdx.x == 0) {
    lse_out[r] = l;
    const uint16_t raw = reinterpret_cast<const uint16_t*>(ce_smem)[y];
    row_loss[r] = l - __uint_as_float((uint32_t)raw << 16);
  }
  // pass 3: dlogits = exp(x - lse) * sc = 2^(x log2e - (lse log2e - log2 sc)), the label's
  // column minus sc afterwards by the thread that wrote its 16-byte group
  const float ob = ce_ob(l, sc);
  if (!GRAD) {
    if (threadIdx.x == 0) ob_out[r] = ob;
    return;
  }
  for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
    const uint4 v = srow[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = pack_bf16(ce_exp(bf_lo(w[e]), ob), ce_exp(bf_hi(w[e]), ob));
    row[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if ((y / 8) % kCeThreads == (int)threadIdx.x) {
    const float xy = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(ce_smem)[y] << 16);
    rowp[y] = __float2bfloat16(ce_exp(xy, ob) - sc);
  }
}

// Per-row CE (target < 0 -> 0) from bf16 or fp32 logits; one 256-thread CTA per row.
template <typename T>
__global__ void ce_rows_kernel(const T* __restrict__ logits, long long ld, const long long* __restrict__ tgt, int V,
                               float* __restrict__ out) {
  const long long r = blockIdx.x;
  const T* x = logits + r * ld;
  __shared__ float red[32];
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, (float)x[i]);
  mx = warp_max(mx);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) s += __expf((float)x[i] - mx);
  s = warp_sum(s);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) t += red[w];
    const long long y = tgt[r];
    out[r] = y < 0 ? 0.f : (mx + logf(t) - (float)x[y]);
  }
}

}  // namespace odp

void ce_forward(torch::Tensor part, int64_t T, torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor labels,
                int64_t M, int64_t G, torch::Tensor lse, torch::Tensor row_loss, torch::Tensor loss_sum,
                torch::Tensor inv_count, c10::optional<torch::Tensor> loss_out,
                c10::optional<torch::Tensor> inv_given) {
  c10::cuda::CUDAGuard guard(logits.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int R = (int)(G * M);
  C10_CUDA_CHECK(odp::launch_pdl((odp::ce_finalize_kernel), dim3((R + 255) / 256), dim3(256), 0, st, reinterpret_cast<const float2*>(part.data_ptr<float>()), (int)T,
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), ldl, sl, labels.data_ptr<int>(), (int)M, (int)G,
      lse.data_ptr<float>(), row_loss.data_ptr<float>(), (long long)M));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  C10_CUDA_CHECK(odp::launch_pdl((odp::group_sum_kernel), dim3((int)G), dim3(256), 0, st, row_loss.data_ptr<float>(), labels.data_ptr<int>(), (int)M,
                                                 loss_sum.data_ptr<float>(), inv_count.data_ptr<float>(),
                                                 loss_out.has_value() ? loss_out->data_ptr<float>() : nullptr,
                                                 inv_given.has_value() ? inv_given->data_ptr<float>() : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void ce_attrs() {
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::ce_fused_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        odp::kCeMaxV * 2));
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::ce_fused_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        odp::kCeMaxV * 2));
    attr = true;
  }
}

// Loss and dlogits in one pass over bf16 logits [G][M][V] (row stride ldl, group stride sl):
// lse, row_loss per row, loss_sum / inv_count / optional per-group mean loss per group;
// logits are overwritten with dlogits = (softmax - onehot) / count. With `ob` the logits are
// only read: ob = ce_ob(lse, 1 / count) per row is written instead, for GEMMs that form the
// dlogits themselves (gemm_ce_grad).
void ce_fused(torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor labels, int64_t M, int64_t V, int64_t G,
              torch::Tensor lse, torch::Tensor row_loss, torch::Tensor loss_sum, torch::Tensor inv_count,
              c10::optional<torch::Tensor> loss_out, torch::Tensor err, c10::optional<torch::Tensor> inv_given,
              c10::optional<torch::Tensor> ob) {
  TORCH_CHECK(V % 8 == 0 && ldl % 8 == 0 && sl % 8 == 0 && V <= odp::kCeMaxV,
              "ce_fused: vocab must be a multiple of 8 and at most 32768");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0, "ce_fused: logits must be 16-byte aligned");
  c10::cuda::CUDAGuard guard(logits.device());
  auto st = at::cuda::getCurrentCUDAStream();
  ce_attrs();
  const float* given = inv_given.has_value() ? inv_given->data_ptr<float>() : nullptr;
  if (!given) {
    C10_CUDA_CHECK(odp::launch_pdl((odp::label_count_kernel), dim3((int)G), dim3(256), 0, st, labels.data_ptr<int>(), (int)M, inv_count.data_ptr<float>()));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  C10_CUDA_CHECK(odp::launch_pdl(ob.has_value() ? odp::ce_fused_kernel<false> : odp::ce_fused_kernel<true>,
                                 dim3((unsigned)(G * M)), dim3(odp::kCeThreads), (size_t)V * 2, st,
                                 reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), ldl, sl,
                                 labels.data_ptr<int>(), (int)M, (int)V,
                                 given ? given : inv_count.data_ptr<float>(), lse.data_ptr<float>(),
                                 row_loss.data_ptr<float>(), err.data_ptr<int>(), (long long)M,
                                 ob.has_value() ? ob->data_ptr<float>() : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  C10_CUDA_CHECK(odp::launch_pdl((odp::group_sum_kernel), dim3((int)G), dim3(256), 0, st, row_loss.data_ptr<float>(), labels.data_ptr<int>(), (int)M,
                                                 loss_sum.data_ptr<float>(), inv_count.data_ptr<float>(),
                                                 loss_out.has_value() ? loss_out->data_ptr<float>() : nullptr, given));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_backward(torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor lse, torch::Tensor labels,
                 torch::Tensor inv_count, int64_t M, int64_t V, int64_t G) {
  TORCH_CHECK(V % 8 == 0 && ldl % 8 == 0, "ce_backward: vocab must be a multiple of 8");
  c10::cuda::CUDAGuard guard(logits.device());
  const long long n = G * M * (V / 8);
  C10_CUDA_CHECK(odp::launch_pdl((odp::ce_backward_kernel), dim3((unsigned)((n + 255) / 256)), dim3(256), 0, at::cuda::getCurrentCUDAStream(), reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), ldl, sl, lse.data_ptr<float>(), labels.data_ptr<int>(),
      inv_count.data_ptr<float>(), (int)M, (int)V, (int)G, (long long)M));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------- row chunks
// The loss over a batch computed in chunks of each group's rows (bounded logits memory):
// ce_label_count once (the dlogits scale needs the whole batch's count), then per chunk
// the GEMM's logits for rows [r0, r0 + Mc) and ce_rows_chunk (labels / lse / row_loss
// passed offset to r0, group stride ms = the batch's rows), and ce_group_sum once over
// all rows at the end.
void ce_label_count(torch::Tensor labels, int64_t M, int64_t G, torch::Tensor inv_count) {
  c10::cuda::CUDAGuard guard(labels.device());
  C10_CUDA_CHECK(odp::launch_pdl((odp::label_count_kernel), dim3((int)G), dim3(256), 0, at::cuda::getCurrentCUDAStream(), labels.data_ptr<int>(), (int)M,
                                                                                 inv_count.data_ptr<float>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_group_sum(torch::Tensor row_loss, torch::Tensor labels, int64_t M, int64_t G, torch::Tensor loss_sum,
                  torch::Tensor inv_count, c10::optional<torch::Tensor> loss_out, c10::optional<torch::Tensor> inv_given) {
  c10::cuda::CUDAGuard guard(labels.device());
  C10_CUDA_CHECK(odp::launch_pdl((odp::group_sum_kernel), dim3((int)G), dim3(256), 0, at::cuda::getCurrentCUDAStream(), row_loss.data_ptr<float>(), labels.data_ptr<int>(), (int)M, loss_sum.data_ptr<float>(),
      inv_count.data_ptr<float>(), loss_out.has_value() ? loss_out->data_ptr<float>() : nullptr,
      inv_given.has_value() ? inv_given->data_ptr<float>() : nullptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One chunk: logits [G][Mc] rows (row stride ldl, group stride sl) -> lse, row losses and
// in-place dlogits scaled by inv (the batch's 1 / count per group). One-pass kernel for
// V <= 32768; wider vocabularies merge the logits GEMM's (max, sum exp) partials
// `part` ([G][Mc][T] float2) and then rewrite the logits.
void ce_rows_chunk(torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor labels, int64_t Mc, int64_t ms,
                   int64_t V, int64_t G, torch::Tensor lse, torch::Tensor row_loss, torch::Tensor inv,
                   c10::optional<torch::Tensor> part, int64_t T, torch::Tensor err, c10::optional<torch::Tensor> ob) {
  TORCH_CHECK(V % 8 == 0 && ldl % 8 == 0 && sl % 8 == 0, "ce_rows_chunk: vocab and strides multiples of 8");
  c10::cuda::CUDAGuard guard(logits.device());
  auto st = at::cuda::getCurrentCUDAStream();
  if (!part.has_value()) {
    TORCH_CHECK(V <= odp::kCeMaxV && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0,
                "ce_rows_chunk: the one-pass kernel takes at most 32768 columns, 16-byte aligned rows");
    ce_attrs();
    C10_CUDA_CHECK(odp::launch_pdl(ob.has_value() ? odp::ce_fused_kernel<false> : odp::ce_fused_kernel<true>,
                                   dim3((unsigned)(G * Mc)), dim3(odp::kCeThreads), (size_t)V * 2, st,
                                   reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), ldl, sl,
                                   labels.data_ptr<int>(), (int)Mc, (int)V, inv.data_ptr<float>(),
                                   lse.data_ptr<float>(), row_loss.data_ptr<float>(), err.data_ptr<int>(), ms,
                                   ob.has_value() ? ob->data_ptr<float>() : nullptr));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  TORCH_CHECK(!ob.has_value(), "ce_rows_chunk: the stats-only form needs the one-pass kernel (V <= 32768)");
  const int R = (int)(G * Mc);
  C10_CUDA_CHECK(odp::launch_pdl((odp::ce_finalize_kernel), dim3((R + 255) / 256), dim3(256), 0, st, reinterpret_cast<const float2*>(part->data_ptr<float>()), (int)T,
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), ldl, sl, labels.data_ptr<int>(), (int)Mc, (int)G,
      lse.data_ptr<float>(), row_loss.data_ptr<float>(), ms));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const long long n = G * Mc * (V / 8);
  C10_CUDA_CHECK(odp::launch_pdl((odp::ce_backward_kernel), dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), ldl, sl, lse.data_ptr<float>(), labels.data_ptr<int>(),
      inv.data_ptr<float>(), (int)Mc, (int)V, (int)G, ms));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

torch::Tensor cross_entropy_rows(torch::Tensor logits, torch::Tensor target) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "cross_entropy_rows: [R, V] row-major logits");
  c10::cuda::CUDAGuard guard(logits.device());
  auto tgt = target.to(torch::kLong).contiguous();
  auto out = torch::empty({logits.size(0)}, logits.options().dtype(torch::kFloat));
  if (logits.size(0) == 0) return out;
  auto st = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kBFloat16) {
    odp::ce_rows_kernel<__nv_bfloat16><<<(unsigned)logits.size(0), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), reinterpret_cast<const long long*>(tgt.data_ptr<int64_t>()),
        (int)logits.size(1), out.data_ptr<float>());
  } else {
    TORCH_CHECK(logits.scalar_type() == at::kFloat, "cross_entropy_rows: bf16 or fp32 logits");
    odp::ce_rows_kernel<float><<<(unsigned)logits.size(0), 256, 0, st>>>(
        logits.data_ptr<float>(), logits.stride(0), reinterpret_cast<const long long*>(tgt.data_ptr<int64_t>()), (int)logits.size(1),
        out.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}
