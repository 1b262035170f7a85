// Device-side input normalisation: per-volume z-score of a uint8 batch into bf16 / fp32.
//
// Volumes arrive from the host as uint8 (a quarter of the bytes of fp32), so the z-score runs on
// the device as two passes over the batch:
//   1. u8_moments_kernel: per-volume sum and sum of squares, accumulated exactly in integers
//      (32-bit per thread, 64-bit atomics per CTA), so the mean and the unbiased variance are exact.
//   2. u8_zscore_kernel: y = (x - mean) / max(std, 1e-6), 16 voxels per thread, written as bf16 or
//      fp32.
// Traffic: the uint8 batch twice plus the output once (134 MB for 16 x 128^3 into bf16).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mia {
namespace {

constexpr int kZThreads = 256;

__global__ void __launch_bounds__(kZThreads) u8_moments_kernel(const uint8_t* __restrict__ x, int64_t per_vol,
                                                               unsigned long long* __restrict__ moments) {
  const int b = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)b * per_vol);
  const int64_t chunks = per_vol / 16;
  uint32_t s = 0;
  unsigned long long q = 0;
  for (int64_t c = (int64_t)blockIdx.x * kZThreads + threadIdx.x; c < chunks; c += (int64_t)gridDim.x * kZThreads) {
    const uint4 u = src[c];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t qs = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t v = (w[i] >> (8 * k)) & 0xFFu;
        s += v;
        qs += v * v;  // <= 16 * 65025, no overflow
      }
    }
    q += qs;
  }
  // tail voxels (per_vol % 16) by the first CTA of the volume
  if (blockIdx.x == 0) {
    for (int64_t i = chunks * 16 + threadIdx.x; i < per_vol; i += kZThreads) {
      const uint32_t v = x[(size_t)b * per_vol + i];
      s += v;
      q += v * v;
    }
  }
  unsigned long long s64 = s;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    s64 += __shfl_xor_sync(0xffffffffu, s64, off);
    q += __shfl_xor_sync(0xffffffffu, q, off);
  }
  __shared__ unsigned long long ws[kZThreads / 32][2];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    ws[warp][0] = s64;
    ws[warp][1] = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long ts = 0, tq = 0;
    for (int w = 0; w < kZThreads / 32; ++w) {
      ts += ws[w][0];
      tq += ws[w][1];
    }
    atomicAdd(&moments[2 * b], ts);
    atomicAdd(&moments[2 * b + 1], tq);
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* dst, const float (&v)[16]);

template <>
__device__ __forceinline__ void store16<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  d[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                    pack_bf16x2(v[14], v[15]));
}

template <>
__device__ __forceinline__ void store16<float>(float* dst, const float (&v)[16]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__device__ __forceinline__ void volume_stats(const unsigned long long* moments, int b, int64_t n, float& mean,
                                             float& inv_std) {
  const double s = (double)moments[2 * b], q = (double)moments[2 * b + 1];
  const double m = s / (double)n;
  const double var = n > 1 ? fmax((q - s * m) / (double)(n - 1), 0.0) : 0.0;
  mean = (float)m;
  inv_std = (float)(1.0 / fmax(sqrt(var), 1e-6));
}

template <typename T>
__global__ void __launch_bounds__(kZThreads) u8_zscore_kernel(const uint8_t* __restrict__ x, int64_t per_vol,
                                                              const unsigned long long* __restrict__ moments,
                                                              T* __restrict__ out) {
  const int b = blockIdx.y;
  float mean, inv_std;
  volume_stats(moments, b, per_vol, mean, inv_std);
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)b * per_vol);
  T* dst = out + (size_t)b * per_vol;
  const int64_t chunks = per_vol / 16;
  for (int64_t c = (int64_t)blockIdx.x * kZThreads + threadIdx.x; c < chunks; c += (int64_t)gridDim.x * kZThreads) {
    const uint4 u = src[c];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float v[16];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) v[4 * i + k] = ((float)((w[i] >> (8 * k)) & 0xFFu) - mean) * inv_std;
    store16<T>(dst + c * 16, v);
  }
  if (blockIdx.x == 0) {
    for (int64_t i = chunks * 16 + threadIdx.x; i < per_vol; i += kZThreads)
      dst[i] = (T)(((float)x[(size_t)b * per_vol + i] - mean) * inv_std);
  }
}

}  // namespace

// x: contiguous uint8 (B, ...); out: contiguous bf16 or fp32 of the same shape.
void zscore_u8(torch::Tensor x, torch::Tensor out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kByte && x.is_contiguous() && x.dim() >= 1,
              "zscore_u8: contiguous uint8 CUDA input");
  TORCH_CHECK(out.is_contiguous() && out.sizes() == x.sizes() &&
                  (out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat),
              "zscore_u8: contiguous bf16 / fp32 output of the input's shape");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "zscore_u8: 16-byte aligned buffers");
  const int B = (int)x.size(0);
  const int64_t per_vol = B > 0 ? x.numel() / B : 0;
  TORCH_CHECK(per_vol % 16 == 0 || B == 1, "zscore_u8: voxels per volume must be a multiple of 16 (or one volume)");
  if (B == 0 || per_vol == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto moments = torch::zeros({B, 2}, x.options().dtype(at::kLong));
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.get_device()));
  const int64_t chunks = std::max<int64_t>(1, per_vol / 16);
  const int gx = (int)std::max<int64_t>(1, std::min<int64_t>((chunks + kZThreads - 1) / kZThreads,
                                                            (int64_t)(4 * sms + B - 1) / B));
  auto* mom = reinterpret_cast<unsigned long long*>(moments.data_ptr<int64_t>());
  u8_moments_kernel<<<dim3(gx, B), kZThreads, 0, stream>>>(x.data_ptr<uint8_t>(), per_vol, mom);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (out.scalar_type() == at::kBFloat16) {
    u8_zscore_kernel<__nv_bfloat16><<<dim3(gx, B), kZThreads, 0, stream>>>(
        x.data_ptr<uint8_t>(), per_vol, mom, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  } else {
    u8_zscore_kernel<float><<<dim3(gx, B), kZThreads, 0, stream>>>(x.data_ptr<uint8_t>(), per_vol, mom,
                                                                   out.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
