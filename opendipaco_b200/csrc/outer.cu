// DiLoCo outer step, fused into one kernel over every shared module a GPU owns.
//
// For each element e of a shared module key k with local sharers j (working copies
// of the paths on this GPU that use k, weights w_j):
//     acc  = sum_j w_j * (global[e] - local_j[e])        (in path order, fp32, no FMA)
//     d    = acc / den_k  (normalize_outer_delta)  * scale_k (sqrt(sharing count))
//     buf  = first ? d : m * buf + d                     (torch SGD momentum buffer)
//     upd  = nesterov ? d + m * buf : buf
//     global[e] -= lr * upd ;  every local_j[e] = global[e] (fp32 + bf16 copy)
// and per-chunk partial sums of d^2 for the delta-norm metric (reduced in a fixed
// order on the host side of the call).
//
// This is the pseudo-gradient, the reduction over the sharing paths, Nesterov and
// the write-back to all sharers' working copies in one pass: each byte of the
// global, momentum and local copies is read and written once. Private modules use
// mode COPY (global = the single local copy, no outer step). The cross-GPU variant
// (peer-memory slice reduction) lives in outer_nvlink.cu.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

struct OuterSeg {
  float* glob;
  float* mom;       // null for COPY
  float* delta;     // ACC writes sum_j w_j (global - local_j) here; APPLY reads it
  long long n;
  int first_local;  // index into the local table
  int nlocal;
  int mode;         // 0 = outer step, 1 = copy local -> global, 2 = broadcast global -> locals,
                    // 3 = accumulate local pseudo-gradient into delta, 4 = apply delta (outer step)
  float scale;      // sqrt(sharing) (or 1)
  float inv_den;    // 1 / sum w  (normalize) or 1
  long long chunk0; // first chunk index of this segment in the flat chunk space
};

struct OuterLocal {
  float* w32;
  __nv_bfloat16* w16;
  float weight;
};

constexpr int kOuterChunk = 4096;

__global__ void outer_step_kernel(const OuterSeg* __restrict__ segs, int nseg, const OuterLocal* __restrict__ locs,
                                  long long total_chunks, float lr, float mom, int nesterov, int first,
                                  float* __restrict__ sq_part) {
  __shared__ float red[8];
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    // binary search the segment owning this chunk
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (segs[mid].chunk0 <= ch) lo = mid;
      else hi = mid - 1;
    }
    const OuterSeg s = segs[lo];
    const long long e0 = (ch - s.chunk0) * kOuterChunk;
    const long long e1 = min(e0 + kOuterChunk, s.n);
    float sq = 0.f;
    for (long long e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
      if (s.mode == 1) {
        s.glob[e] = locs[s.first_local].w32[e];
        continue;
      }
      if (s.mode == 2) {
        const float gv = s.glob[e];
        for (int j = 0; j < s.nlocal; ++j) {
          const OuterLocal L = locs[s.first_local + j];
          L.w32[e] = gv;
          if (L.w16) L.w16[e] = __float2bfloat16(gv);
        }
        continue;
      }
      const float gv = s.glob[e];
      float acc = 0.f;
      if (s.mode == 4) {
        acc = s.delta[e];
      } else {
        for (int j = 0; j < s.nlocal; ++j) {
          const OuterLocal L = locs[s.first_local + j];
          acc = __fadd_rn(acc, __fmul_rn(L.weight, __fsub_rn(gv, L.w32[e])));
        }
        if (s.mode == 3) {
          s.delta[e] = acc;
          continue;
        }
      }
      float d = __fmul_rn(__fmul_rn(acc, s.inv_den), s.scale);
      sq += d * d;
      float b = first ? d : __fadd_rn(__fmul_rn(s.mom[e], mom), d);
      s.mom[e] = b;
      const float upd = nesterov ? __fadd_rn(d, __fmul_rn(mom, b)) : b;
      const float ng = __fadd_rn(gv, __fmul_rn(-lr, upd));
      s.glob[e] = ng;
      for (int j = 0; j < s.nlocal; ++j) {
        const OuterLocal L = locs[s.first_local + j];
        L.w32[e] = ng;
        if (L.w16) L.w16[e] = __float2bfloat16(ng);
      }
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

}  // namespace odp

// segs: int64 tensor [nseg, 10] packed on the host (pointers, sizes, floats as bits);
// locals: int64 tensor [nloc, 3]. Both must live on the device.
void outer_step(torch::Tensor segs, int64_t nseg, torch::Tensor locals, int64_t total_chunks, double lr,
                double momentum, bool nesterov, bool first, c10::optional<torch::Tensor> sq_part) {
  static_assert(sizeof(odp::OuterSeg) == 64, "OuterSeg layout");
  static_assert(sizeof(odp::OuterLocal) == 24, "OuterLocal layout");
  TORCH_CHECK(segs.is_cuda() && locals.is_cuda(), "outer_step: tables must be on the device");
  c10::cuda::CUDAGuard guard(segs.device());
  if (total_chunks == 0) return;
  const int grid = (int)std::min<int64_t>(total_chunks, 148 * 8);
  odp::outer_step_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::OuterSeg*>(segs.data_ptr()), (int)nseg,
      reinterpret_cast<const odp::OuterLocal*>(locals.data_ptr()), total_chunks, (float)lr, (float)momentum,
      nesterov ? 1 : 0, first ? 1 : 0, sq_part.has_value() ? sq_part->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t outer_chunk_elems() { return odp::kOuterChunk; }
