// Wire-compression codecs and robust aggregation on the GPU.
//
// quant_int4: symmetric int4 with one scale per group of 128 (scale = absmax / 7,
//   q = rint(x / scale) clamped to [-7, 7], stored as q + 8 with two values per byte,
//   high nibble first) and the error-feedback residual x - q * scale, in one pass:
//   one warp per group, 4 consecutive values per lane.
// dequant_int4: the inverse, optionally fused into "dst += w * x" (decode straight
//   into an accumulator, no fp32 staging copy).
// quant_int8: per-tensor symmetric int8 (absmax / 127) + residual; the absmax is a
//   deterministic two-stage reduction.
// robust_combine: coordinate-wise mean / trimmed mean (drop min and max when >= 3)
//   / lower median over c <= 16 stacked contributions (register insertion sort).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

__global__ void quant_int4_kernel(const float* __restrict__ x, long long n, uint8_t* __restrict__ packed,
                                  float* __restrict__ scale, float* __restrict__ resid, long long ngroups, int vec) {
  const long long grp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (grp >= ngroups) return;
  const long long e0 = grp * 128 + lane * 4;
  const bool full = vec && e0 + 4 <= n;  // one 16-byte load and store per lane
  float v[4];
  if (full) {
    const float4 a = *reinterpret_cast<const float4*>(x + e0);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = e0 + i < n ? x[e0 + i] : 0.f;
  }
  float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  am = warp_max(am);
  const float s = am / 7.0f;
  const float safe = s > 0.f ? s : 1.f;
  int q[4];
  float r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    q[i] = (int)fminf(fmaxf(rintf(v[i] / safe), -7.f), 7.f);
    r[i] = v[i] - __fmul_rn((float)q[i], s);  // no FMA: same rounding as the host
  }
  if (resid) {
    if (full) {
      *reinterpret_cast<float4*>(resid + e0) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (e0 + i < n) resid[e0 + i] = r[i];
    }
  }
  const uint16_t two = (uint16_t)((((q[0] + 8) << 4) | (q[1] + 8)) | ((((q[2] + 8) << 4) | (q[3] + 8)) << 8));
  *reinterpret_cast<uint16_t*>(packed + grp * 64 + lane * 2) = two;  // bytes in order: (q0 q1), (q2 q3)
  if (lane == 0) scale[grp] = s;
}

__global__ void dequant_int4_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ scale,
                                    long long n, int g, float* __restrict__ out, float w, int accumulate) {
  const long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // byte index
  const long long e = 2 * j;
  if (e >= n) return;
  const uint8_t b = packed[j];
  const float s = scale[e / g];
  const float v0 = (float)((b >> 4) & 15) - 8.f, v1 = (float)(b & 15) - 8.f;
  if (accumulate) {
    out[e] += w * (v0 * s);
    if (e + 1 < n) out[e + 1] += w * (v1 * s);
  } else {
    out[e] = v0 * s;
    if (e + 1 < n) out[e + 1] = v1 * s;
  }
}

__global__ void absmax_part_kernel(const float* __restrict__ x, long long n, float* __restrict__ part) {
  float m = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  __shared__ float red[32];
  m = warp_max(m);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < (int)blockDim.x / 32; ++k) t = fmaxf(t, red[k]);
    part[blockIdx.x] = t;
  }
}

__global__ void quant_int8_kernel(const float* __restrict__ x, long long n, const float* __restrict__ part, int nparts,
                                  int8_t* __restrict__ q, float* __restrict__ resid, float* __restrict__ scale_out) {
  float am = 0.f;
  for (int k = 0; k < nparts; ++k) am = fmaxf(am, part[k]);
  const float s = (float)((double)am / 127.0);
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = am;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i];
    int qi = 0;
    if (s != 0.f) qi = (int)fminf(fmaxf(rintf(v / s), -127.f), 127.f);
    q[i] = (int8_t)qi;
    if (resid) resid[i] = s != 0.f ? v - __fmul_rn((float)qi, s) : v;  // no FMA: same rounding as the host
  }
}

// stack: [c][n] fp32; mode 0 mean, 1 trimmed mean, 2 median (lower middle).
__global__ void robust_combine_kernel(const float* __restrict__ stack, int c, long long n, int mode,
                                      float* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v[16];
  for (int k = 0; k < c; ++k) {
    float x = stack[(long long)k * n + i];
    int j = k - 1;
    while (j >= 0 && v[j] > x) {
      v[j + 1] = v[j];
      --j;
    }
    v[j + 1] = x;
  }
  if (mode == 2) {
    out[i] = v[(c - 1) / 2];
    return;
  }
  int lo = 0, hi = c;
  if (mode == 1 && c >= 3) {
    lo = 1;
    hi = c - 1;
  }
  float s = 0.f;
  for (int k = lo; k < hi; ++k) s += v[k];
  out[i] = s / (float)(hi - lo);
}

}  // namespace odp

static int nblk(long long n, int per) { return (int)((n + per - 1) / per); }

std::vector<torch::Tensor> quant_int4(torch::Tensor x, bool want_resid) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat, "quant_int4: fp32 CUDA tensor");
  c10::cuda::CUDAGuard guard(x.device());
  auto xf = x.contiguous().view(-1);
  const long long n = xf.numel(), ng = (n + 127) / 128;
  auto packed = torch::empty({ng * 64}, x.options().dtype(torch::kUInt8));
  auto scale = torch::empty({ng}, x.options());
  auto resid = want_resid ? torch::empty_like(xf) : torch::Tensor();
  if (ng)
    odp::quant_int4_kernel<<<nblk(ng * 32, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        xf.data_ptr<float>(), n, packed.data_ptr<uint8_t>(), scale.data_ptr<float>(),
        want_resid ? resid.data_ptr<float>() : nullptr, ng,
        reinterpret_cast<uintptr_t>(xf.data_ptr()) % 16 == 0 &&
                (!want_resid || reinterpret_cast<uintptr_t>(resid.data_ptr()) % 16 == 0)
            ? 1
            : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {packed, scale, want_resid ? resid.view(x.sizes()) : resid};
}

void dequant_int4(torch::Tensor packed, torch::Tensor scale, int64_t n, int64_t g, torch::Tensor out, double w,
                  bool accumulate) {
  c10::cuda::CUDAGuard guard(out.device());
  const long long nbytes = (n + 1) / 2;
  if (nbytes)
    odp::dequant_int4_kernel<<<nblk(nbytes, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        packed.data_ptr<uint8_t>(), scale.data_ptr<float>(), n, (int)g, out.data_ptr<float>(), (float)w,
        accumulate ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

std::vector<torch::Tensor> quant_int8(torch::Tensor x, bool want_resid) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat, "quant_int8: fp32 CUDA tensor");
  c10::cuda::CUDAGuard guard(x.device());
  auto xf = x.contiguous().view(-1);
  const long long n = xf.numel();
  const int parts = (int)std::max<long long>(1, std::min<long long>(296, (n + 4095) / 4096));
  auto part = torch::zeros({parts}, x.options());
  auto q = torch::empty({n}, x.options().dtype(torch::kInt8));
  auto resid = want_resid ? torch::empty_like(xf) : torch::Tensor();
  auto amax = torch::zeros({1}, x.options());
  auto st = at::cuda::getCurrentCUDAStream();
  if (n) {
    odp::absmax_part_kernel<<<parts, 256, 0, st>>>(xf.data_ptr<float>(), n, part.data_ptr<float>());
    odp::quant_int8_kernel<<<parts, 256, 0, st>>>(xf.data_ptr<float>(), n, part.data_ptr<float>(), parts,
                                                   q.data_ptr<int8_t>(), want_resid ? resid.data_ptr<float>() : nullptr,
                                                   amax.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q.view(x.sizes()), amax, want_resid ? resid.view(x.sizes()) : resid};
}

torch::Tensor robust_combine(torch::Tensor stack, int64_t mode) {
  TORCH_CHECK(stack.is_cuda() && stack.scalar_type() == at::kFloat && stack.size(0) <= 16,
              "robust_combine: fp32 CUDA [c<=16, ...]");
  c10::cuda::CUDAGuard guard(stack.device());
  auto s = stack.contiguous();
  const int c = (int)s.size(0);
  const long long n = s.numel() / c;
  auto out = torch::empty(s.sizes().slice(1), s.options());
  if (n)
    odp::robust_combine_kernel<<<nblk(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        s.data_ptr<float>(), c, n, (int)mode, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}
