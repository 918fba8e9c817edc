// Intra-path data parallelism over NVLink peer memory: one path's batch is split over a
// group of d GPUs (one process each). The group's fp32 master weights, bf16 working
// copies, gradients and AdamW moments live in symmetric buffers (the same offsets on
// every member), so after each inner step's backward the group finishes the step with
// kernels that address each other's memory directly, no NCCL:
//
//   dp_barrier      every member has finished writing what the others will read next
//   dp_grad_reduce  member j sums the d members' gradients (peer loads, fixed member
//                   order, so every run adds in the same order) over its shard
//                   [j * PS, (j + 1) * PS) of every path's flat vector, writes the sum
//                   into its own GRAD shard and per-block sums of squares
//   dp_norm         each member publishes its per-path shard sum of squares to every
//                   member, waits for all, and derives the clip coefficient from the
//                   global norm (torch.nn.utils.clip_grad_norm_ semantics)
//   dp_adamw        AdamW (decoupled weight decay, bias-corrected moments) on the shard,
//                   storing the new fp32 master, its bf16 copy and both moments into
//                   EVERY member's buffers: the reduce-scatter is fused with the update
//                   and the all-gather is fused into the update's stores
//   dp_adam8bit     the same with blockwise 8-bit Adam (blocks of 256 never straddle a
//                   shard): the requantised moments, their scales and the new weights are
//                   stored into every member
//   dp_barrier      before the next forward reads the gathered weights
//
// Barriers compare monotonically increasing per-member counters kept in device memory,
// so the sequence is valid inside a CUDA graph replayed many times. Every wait is
// bounded by the launch argument `bound_ns` (peer_wait_bound_ns, 2 s by default): on
// timeout the kernel records ERR_TIMEOUT_PEER and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {
namespace dp {

constexpr int kMaxMembers = 8;
constexpr int kBlockElems = 1 << 16;  // sum-of-squares partial granularity

// Device pointer table (int64): rows W32, W16, GRAD, M1, M2, PAD, NORM and the 8-bit Adam
// state MQ, MABS, VQ, VLO, VSC; kMaxMembers each (unused rows are 0).
enum Row {
  W32 = 0, W16 = 1, GRAD = 2, M1 = 3, M2 = 4, PAD = 5, NORM = 6,
  MQ = 7, MABS = 8, VQ = 9, VLO = 10, VSC = 11, NROWS = 12
};

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

template <typename T>
ODP_DEVICE T* row_ptr(const long long* tab, int row, int member) {
  return reinterpret_cast<T*>(tab[row * kMaxMembers + member]);
}

// Thread 0 only. pad (uint32 [kMaxMembers]) of every member holds the last counter value
// each member published; counter (uint32, this member's device memory) counts barriers.
ODP_DEVICE bool group_barrier(const long long* tab, unsigned* counter, int me, int d, int* err,
                              unsigned long long bound_ns) {
  const unsigned v = *counter + 1;
  *counter = v;
  __threadfence_system();  // this member's earlier peer and local stores precede the signal
  for (int p = 0; p < d; ++p) st_release_sys(row_ptr<unsigned>(tab, PAD, p) + me, v);
  const unsigned* mine = row_ptr<const unsigned>(tab, PAD, me);
  const unsigned long long t0 = globaltimer();
  for (int p = 0; p < d; ++p) {
    while ((int)(ld_acquire_sys(mine + p) - v) < 0) {
      if (globaltimer() - t0 > bound_ns) {
        record_error(err, ERR_TIMEOUT_PEER);
        return false;
      }
    }
  }
  return true;
}

__global__ void barrier_kernel(const long long* tab, unsigned* counter, int me, int d, int* err,
                               unsigned long long bound_ns) {
  if (threadIdx.x == 0) group_barrier(tab, counter, me, d, err, bound_ns);
}

// grid (nblk, G): block b of path g covers [s0 + b * kBlockElems, ...) of the shard.
__global__ void __launch_bounds__(256) grad_reduce_kernel(const long long* tab, int me, int d, long long P,
                                                           long long stride, long long s0, long long s1, int nblk,
                                                           float* __restrict__ part) {
  const int g = blockIdx.y, b = blockIdx.x;
  const long long e0 = s0 + (long long)b * kBlockElems;
  const long long e1 = min(e0 + kBlockElems, s1);
  float* own = row_ptr<float>(tab, GRAD, me) + g * stride;
  float sq = 0.f;
  for (long long e = e0 + threadIdx.x * 4; e < e1; e += 256 * 4) {
    float4 acc = ld_cg4(row_ptr<const float>(tab, GRAD, 0) + g * stride + e);
    for (int p = 1; p < d; ++p) {
      const float4 x = ld_cg4(row_ptr<const float>(tab, GRAD, p) + g * stride + e);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    *reinterpret_cast<float4*>(own + e) = acc;
    sq += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  __shared__ float red[8];
  sq = warp_sum(sq);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    part[(long long)g * nblk + b] = t;
  }
}

// One CTA: shard sums of squares -> every member's NORM[me][g]; barrier; global norm.
__global__ void __launch_bounds__(256) norm_kernel(const long long* tab, unsigned* counter, int me, int d, int G,
                                                    const float* __restrict__ part, int nblk, float max_norm,
                                                    float* __restrict__ coef, float* __restrict__ gnorm, int* err,
                                                    unsigned long long bound_ns) {
  __shared__ float red[256];
  __shared__ int ok;
  for (int g = 0; g < G; ++g) {
    float s = 0.f;
    for (int i = threadIdx.x; i < nblk; i += 256) s += part[(long long)g * nblk + i];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x < d) row_ptr<float>(tab, NORM, threadIdx.x)[me * G + g] = red[0];
    __syncthreads();
  }
  if (threadIdx.x == 0) ok = group_barrier(tab, counter, me, d, err, bound_ns) ? 1 : 0;
  __syncthreads();
  if (!ok) return;
  const float* mine = row_ptr<const float>(tab, NORM, me);
  for (int g = threadIdx.x; g < G; g += 256) {
    float s = 0.f;
    for (int p = 0; p < d; ++p) s += *reinterpret_cast<const volatile float*>(mine + p * G + g);
    const float n = sqrtf(s);
    gnorm[g] = n;
    coef[g] = max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
  }
}

// grid (ceil((s1 - s0) / 1024), G). sched: [G][4] = lr, lr / bc1, sqrt(bc2), active.
__global__ void __launch_bounds__(256) adamw_kernel(const long long* tab, int me, int d, long long stride,
                                                     long long stride16, long long s0, long long s1,
                                                     const float* __restrict__ coef, const float* __restrict__ sched,
                                                     float b1, float b2, float eps, float wd) {
  const int g = blockIdx.y;
  const long long e = s0 + ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (e >= s1) return;
  const float* sc = sched + g * 4;
  if (sc[3] == 0.f) return;  // path without data this step: untouched everywhere
  const float lr = sc[0], step_size = sc[1], bc2s = sc[2], cf = coef[g];
  const long long o = g * stride + e, o16 = g * stride16 + e;
  const float4 p = *reinterpret_cast<const float4*>(row_ptr<const float>(tab, W32, me) + o);
  const float4 gr = *reinterpret_cast<const float4*>(row_ptr<const float>(tab, GRAD, me) + o);
  const float4 m = *reinterpret_cast<const float4*>(row_ptr<const float>(tab, M1, me) + o);
  const float4 v = *reinterpret_cast<const float4*>(row_ptr<const float>(tab, M2, me) + o);
  const float pi[4] = {p.x, p.y, p.z, p.w}, gi[4] = {gr.x, gr.y, gr.z, gr.w};
  const float mi[4] = {m.x, m.y, m.z, m.w}, vi[4] = {v.x, v.y, v.z, v.w};
  float po[4], mo[4], vo[4];
  const float decay = 1.f - lr * wd;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float gg = gi[i] * cf;
    mo[i] = b1 * mi[i] + (1.f - b1) * gg;
    vo[i] = b2 * vi[i] + (1.f - b2) * gg * gg;
    const float den = sqrtf(vo[i]) / bc2s + eps;
    po[i] = pi[i] * decay - step_size * (mo[i] / den);
  }
  const float4 P4 = make_float4(po[0], po[1], po[2], po[3]);
  const float4 M4 = make_float4(mo[0], mo[1], mo[2], mo[3]);
  const float4 V4 = make_float4(vo[0], vo[1], vo[2], vo[3]);
  const uint2 B4 = make_uint2(pack_bf16(po[0], po[1]), pack_bf16(po[2], po[3]));
  for (int q = 0; q < d; ++q) {  // every member, this one included: the fused all-gather
    *reinterpret_cast<float4*>(row_ptr<float>(tab, W32, q) + o) = P4;
    *reinterpret_cast<float4*>(row_ptr<float>(tab, M1, q) + o) = M4;
    *reinterpret_cast<float4*>(row_ptr<float>(tab, M2, q) + o) = V4;
    *reinterpret_cast<uint2*>(row_ptr<__nv_bfloat16>(tab, W16, q) + o16) = B4;
  }
}

// One warp per 256-element block of the shard: grid covers G * nbs warps, nbs = blocks per
// path in the shard, block b of path g is global block g * nb + b0 + b. Same update as the
// single-GPU adam8bit kernel (int8 absmax m, log-domain uint8 v, round half to even).
__global__ void adam8bit_kernel(const long long* tab, int me, int d, int G, long long P, long long nb, long long b0,
                                long long nbs, const float* __restrict__ coef, const float* __restrict__ sched,
                                float b1, float b2, float eps, float wd) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= (long long)G * nbs) return;
  const int g = (int)(w / nbs);
  const long long blk = (long long)g * nb + b0 + (w % nbs);
  const float* scd = sched + g * 4;
  if (scd[3] == 0.f) return;
  const float lr = scd[0], step_size = scd[1], bc2s = scd[2];
  const bool first_step = scd[3] > 1.5f;
  const float cf = coef[g];
  const long long e0 = (long long)g * P + (b0 + (w % nbs)) * 256 + lane * 8;  // element offset in [G][P]
  const long long q0 = blk * 256 + lane * 8;                                  // offset in the [G*nb][256] state
  const float* gr = row_ptr<const float>(tab, GRAD, me);
  const float* pw = row_ptr<const float>(tab, W32, me);
  const int8_t* mq = row_ptr<const int8_t>(tab, MQ, me);
  const uint8_t* vq = row_ptr<const uint8_t>(tab, VQ, me);
  const float mscale = row_ptr<const float>(tab, MABS, me)[blk] / 127.f;
  const float lo = row_ptr<const float>(tab, VLO, me)[blk], vsc = row_ptr<const float>(tab, VSC, me)[blk];
  // every load of the lane in flight at once (16-byte gradient / weight loads, 8-byte codes)
  const float4 g0 = *reinterpret_cast<const float4*>(gr + e0), g1 = *reinterpret_cast<const float4*>(gr + e0 + 4);
  const float4 w0 = *reinterpret_cast<const float4*>(pw + e0), w1 = *reinterpret_cast<const float4*>(pw + e0 + 4);
  const uint2 mcode = *reinterpret_cast<const uint2*>(mq + q0), vcode = *reinterpret_cast<const uint2*>(vq + q0);
  const float gin[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float win[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const int8_t* mc = reinterpret_cast<const int8_t*>(&mcode);
  const uint8_t* vc = reinterpret_cast<const uint8_t*>(&vcode);
  float mv[8], vv[8], lv[8];
  float amax = 0.f, lmin = INFINITY, lmax = -INFINITY;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float gv = gin[k] * cf;
    const float m0 = (float)mc[k] * mscale;
    const float v0 = first_step ? 0.f : __expf((float)vc[k] * vsc + lo);
    mv[k] = m0 * b1 + (1.f - b1) * gv;
    vv[k] = v0 * b2 + (1.f - b2) * gv * gv;
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
  uint32_t mo[2] = {0, 0}, vo[2] = {0, 0};
  float po[8];
  const float decay = 1.f - lr * wd;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t mb = (uint32_t)(uint8_t)(int8_t)fminf(fmaxf(rintf(mv[k] / qs), -127.f), 127.f);
    const uint32_t vb = (uint32_t)(uint8_t)fminf(fmaxf(rintf((lv[k] - lmin) / vs), 0.f), 255.f);
    mo[k / 4] |= mb << (8 * (k % 4));
    vo[k / 4] |= vb << (8 * (k % 4));
    const float den = sqrtf(vv[k]) / bc2s + eps;
    po[k] = win[k] * decay - step_size * (mv[k] / den);
  }
  const float4 p0 = make_float4(po[0], po[1], po[2], po[3]), p1 = make_float4(po[4], po[5], po[6], po[7]);
  const uint4 b16 = make_uint4(pack_bf16(po[0], po[1]), pack_bf16(po[2], po[3]), pack_bf16(po[4], po[5]),
                               pack_bf16(po[6], po[7]));
  for (int q = 0; q < d; ++q) {  // every member, this one included
    float4* pd = reinterpret_cast<float4*>(row_ptr<float>(tab, W32, q) + e0);
    pd[0] = p0;
    pd[1] = p1;
    *reinterpret_cast<uint4*>(row_ptr<__nv_bfloat16>(tab, W16, q) + e0) = b16;
    *reinterpret_cast<uint2*>(row_ptr<int8_t>(tab, MQ, q) + q0) = make_uint2(mo[0], mo[1]);
    *reinterpret_cast<uint2*>(row_ptr<uint8_t>(tab, VQ, q) + q0) = make_uint2(vo[0], vo[1]);
    if (lane == 0) {
      row_ptr<float>(tab, MABS, q)[blk] = amax;
      row_ptr<float>(tab, VLO, q)[blk] = lmin;
      row_ptr<float>(tab, VSC, q)[blk] = vs;
    }
  }
}

}  // namespace dp
}  // namespace odp

static const long long* tab_ptr(torch::Tensor tab) {
  TORCH_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.numel() == odp::dp::NROWS * odp::dp::kMaxMembers,
              "dp: pointer table must be int64 [12][8] on the device");
  return reinterpret_cast<const long long*>(tab.data_ptr<int64_t>());
}

void dp_barrier(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, torch::Tensor err) {
  TORCH_CHECK(d >= 1 && d <= odp::dp::kMaxMembers && me >= 0 && me < d, "dp_barrier: bad group");
  odp::dp::barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      tab_ptr(tab), reinterpret_cast<unsigned*>(counter.data_ptr<int>()), (int)me, (int)d, err.data_ptr<int>(),
      odp::peer_wait_bound_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Reduce-scatter of the gradients + clip coefficient (shard [s0, s1) of G paths of P
// elements, row strides `stride`); `part` holds G * nblk floats of scratch.
void dp_grad_reduce_norm(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, int64_t G, int64_t P,
                         int64_t stride, int64_t s0, int64_t s1, torch::Tensor part, double max_norm,
                         torch::Tensor coef, torch::Tensor gnorm, torch::Tensor err) {
  TORCH_CHECK(s0 % 4 == 0 && s1 % 4 == 0 && stride % 4 == 0 && s1 <= P && s0 <= s1, "dp: shard must be 4-aligned");
  const int nblk = (int)std::max<int64_t>(1, (s1 - s0 + odp::dp::kBlockElems - 1) / odp::dp::kBlockElems);
  TORCH_CHECK(part.numel() >= G * nblk, "dp: partial buffer too small");
  auto st = at::cuda::getCurrentCUDAStream();
  const long long* t = tab_ptr(tab);
  unsigned* cnt = reinterpret_cast<unsigned*>(counter.data_ptr<int>());
  odp::dp::barrier_kernel<<<1, 32, 0, st>>>(t, cnt, (int)me, (int)d, err.data_ptr<int>(), odp::peer_wait_bound_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  odp::dp::grad_reduce_kernel<<<dim3(nblk, (unsigned)G), 256, 0, st>>>(t, (int)me, (int)d, P, stride, s0, s1, nblk,
                                                                       part.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  odp::dp::norm_kernel<<<1, 256, 0, st>>>(t, cnt, (int)me, (int)d, (int)G, part.data_ptr<float>(), nblk,
                                           (float)max_norm, coef.data_ptr<float>(), gnorm.data_ptr<float>(),
                                           err.data_ptr<int>(), odp::peer_wait_bound_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// AdamW on the shard with stores into every member, then the closing barrier.
void dp_adamw(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, int64_t G, int64_t stride,
              int64_t stride16, int64_t s0, int64_t s1, torch::Tensor coef, torch::Tensor sched, double b1, double b2,
              double eps, double wd, torch::Tensor err) {
  auto st = at::cuda::getCurrentCUDAStream();
  const long long* t = tab_ptr(tab);
  if (s1 > s0) {
    const unsigned nb = (unsigned)((s1 - s0 + 1023) / 1024);
    odp::dp::adamw_kernel<<<dim3(nb, (unsigned)G), 256, 0, st>>>(t, (int)me, (int)d, stride, stride16, s0, s1,
                                                                 coef.data_ptr<float>(), sched.data_ptr<float>(),
                                                                 (float)b1, (float)b2, (float)eps, (float)wd);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  odp::dp::barrier_kernel<<<1, 32, 0, st>>>(t, reinterpret_cast<unsigned*>(counter.data_ptr<int>()), (int)me,
                                            (int)d, err.data_ptr<int>(), odp::peer_wait_bound_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// 8-bit Adam on the shard (s0, s1 multiples of 256) with stores into every member, then
// the closing barrier.
void dp_adam8bit(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, int64_t G, int64_t P, int64_t s0,
                 int64_t s1, torch::Tensor coef, torch::Tensor sched, double b1, double b2, double eps, double wd,
                 torch::Tensor err) {
  TORCH_CHECK(P % 256 == 0 && s0 % 256 == 0 && (s1 % 256 == 0 || s1 == P), "dp_adam8bit: 256-element blocks");
  auto st = at::cuda::getCurrentCUDAStream();
  const long long* t = tab_ptr(tab);
  const long long nb = P / 256, b0 = s0 / 256, nbs = (s1 - s0 + 255) / 256;
  if (nbs > 0) {
    const long long warps = G * nbs;
    odp::dp::adam8bit_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
        t, (int)me, (int)d, (int)G, P, nb, b0, nbs, coef.data_ptr<float>(), sched.data_ptr<float>(), (float)b1,
        (float)b2, (float)eps, (float)wd);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  odp::dp::barrier_kernel<<<1, 32, 0, st>>>(t, reinterpret_cast<unsigned*>(counter.data_ptr<int>()), (int)me,
                                            (int)d, err.data_ptr<int>(), odp::peer_wait_bound_ns());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
