// Pull copies over NVLink: one launch moves a list of fp32 segments whose sources may be
// other GPUs' memory (peer pointers of symmetric allocations). Plain 16-byte loads with
// .cg (no L1 allocation) and plain stores; no TMA, so no multicast anywhere. Used for the
// full-bank gather (every module of the bank onto every rank) and for filling the
// momentum slices other ranks own before a checkpoint.
//
// table: int64 [nseg][3] = (source address, destination address, elements). Both
// addresses are 16-byte aligned; a segment's last n % 4 elements are copied one by one.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

__global__ void __launch_bounds__(256) peer_copy_kernel(const long long* __restrict__ tab) {
  const int s = blockIdx.y;
  const float* src = reinterpret_cast<const float*>(tab[3 * s]);
  float* dst = reinterpret_cast<float*>(tab[3 * s + 1]);
  const long long n = tab[3 * s + 2];
  const long long n4 = n >> 2;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  long long i = t0;
  // two loads in flight per thread before the stores
  for (; i + stride < n4; i += 2 * stride) {
    const float4 a = __ldcg(s4 + i), b = __ldcg(s4 + i + stride);
    d4[i] = a;
    d4[i + stride] = b;
  }
  for (; i < n4; i += stride) d4[i] = __ldcg(s4 + i);
  for (long long j = (n4 << 2) + t0; j < n; j += stride) dst[j] = __ldcg(src + j);
}

}  // namespace odp

void peer_copy(torch::Tensor table, int64_t max_elems) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == torch::kLong && table.dim() == 2 && table.size(1) == 3 &&
                  table.is_contiguous(),
              "peer_copy: table is a contiguous int64 [nseg, 3] CUDA tensor");
  const long long nseg = table.size(0);
  if (nseg == 0 || max_elems <= 0) return;
  TORCH_CHECK(nseg <= 65535, "peer_copy: at most 65535 segments per launch");
  c10::cuda::CUDAGuard guard(table.device());
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const long long want = (max_elems / 4 + 255) / 256;
  const unsigned gx = (unsigned)std::max<long long>(1, std::min<long long>(want, std::max<long long>(1, 4 * sms / nseg + 1)));
  odp::peer_copy_kernel<<<dim3(gx, (unsigned)nseg), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const long long*>(table.data_ptr<int64_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
