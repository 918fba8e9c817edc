// DiLoCo outer step on one GPU, fused into one kernel over every module the GPU owns.
//
// For each shared module key k with local sharers j (the working copies of the paths on
// this GPU that use k, weights w_j), per element: the pseudo-gradient sum
// sum_j w_j (global - local_j) (or the one the last inner step's optimizer kernel already
// accumulated), normalisation and sqrt(sharing) scale, the SGD-Nesterov update of the
// global with its momentum, and the write-back of the new global into every sharer's fp32
// and bf16 working copies -- each byte of the global, momentum, pseudo-gradient and local
// copies read and written once (outer_common.cuh has the per-element arithmetic and the
// non-finite guard). Private modules use mode COPY (global = the single local copy). Also
// serves the ACC / APPLY phases of the NCCL baseline (outer step split around an
// all-reduce). The reference computes the same update with eager tensor ops and
// torch.optim.SGD (src/opendipaco/train/loop.py:302-345).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "outer_common.cuh"

namespace odp {

__global__ void __launch_bounds__(256) outer_step_kernel(const OuterSeg* __restrict__ segs, int nseg,
                                                         const OuterLocal* __restrict__ locs, long long total_chunks,
                                                         float lr, float mom, int nesterov, int first,
                                                         float* __restrict__ sq_part, int* status) {
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    const OuterSeg s = segs[find_seg(segs, nseg, ch)];
    const long long e0 = (ch - s.chunk0) * kOuterChunk;
    const long long e1 = min(e0 + kOuterChunk, s.n);
    float sq = 0.f;
    int bad = 0;
    outer_chunk(s, locs, e0, e1, lr, mom, nesterov, first, sq, bad);
    outer_chunk_reduce(sq, bad, ch, sq_part, status);
  }
}

}  // namespace odp

// segs: int64 tensor [nseg, 8] (OuterSeg records); locals: int64 tensor [nloc, 3]
// (OuterLocal records). Both on the device. status: int32 word that counts skipped
// non-finite elements (may be absent).
void outer_step(torch::Tensor segs, int64_t nseg, torch::Tensor locals, int64_t total_chunks, double lr,
                double momentum, bool nesterov, bool first, c10::optional<torch::Tensor> sq_part,
                c10::optional<torch::Tensor> status) {
  static_assert(sizeof(odp::OuterSeg) == 64, "OuterSeg layout");
  static_assert(sizeof(odp::OuterLocal) == 24, "OuterLocal layout");
  TORCH_CHECK(segs.is_cuda() && locals.is_cuda(), "outer_step: tables must be on the device");
  c10::cuda::CUDAGuard guard(segs.device());
  if (total_chunks == 0) return;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const int grid = (int)std::min<int64_t>(total_chunks, (int64_t)sms * 8);
  odp::outer_step_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const odp::OuterSeg*>(segs.data_ptr()), (int)nseg,
      reinterpret_cast<const odp::OuterLocal*>(locals.data_ptr()), total_chunks, (float)lr, (float)momentum,
      nesterov ? 1 : 0, first ? 1 : 0, sq_part.has_value() ? sq_part->data_ptr<float>() : nullptr,
      status.has_value() ? status->data_ptr<int>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t outer_chunk_elems() { return odp::kOuterChunk; }
