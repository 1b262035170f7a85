// Masked-autoencoding kernels: patch gather (the patch-embedding GEMM's A operand), mask-token
// re-insertion and its backward, and the fused norm-pix MSE loss with its gradient.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mia {

typedef __nv_bfloat16 bf16;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// One CTA per (b, kept patch). Row layout (channel, pd, ph, pw) = Conv3d weight flattening.
template <typename Tin, typename Tout>
__global__ void patch_gather_kernel(const Tin* __restrict__ vol, const int64_t* __restrict__ index,
                                    Tout* __restrict__ out, int C, int D, int H, int W, int pd, int ph, int pw, int K) {
  const int row = blockIdx.x;  // b * K + k
  const int b = row / K;
  const int gh = H / ph, gw = W / pw;
  const int64_t p = index[row];
  const int zd = (int)(p / ((int64_t)gh * gw));
  const int zh = (int)((p / gw) % gh);
  const int zw = (int)(p % gw);
  const int vol_patch = pd * ph * pw;
  const int len = C * vol_patch;
  Tout* dst = out + (size_t)row * len;
  for (int e = threadIdx.x; e < len; e += blockDim.x) {
    const int c = e / vol_patch;
    int r = e % vol_patch;
    const int i = r / (ph * pw);
    r %= ph * pw;
    const int j = r / pw, l = r % pw;
    const size_t src = ((((size_t)b * C + c) * D + (zd * pd + i)) * H + (zh * ph + j)) * W + (zw * pw + l);
    dst[e] = from_f<Tout>(to_f<Tin>(vol[src]));
  }
}

void patch_gather(torch::Tensor vol, torch::Tensor index, torch::Tensor out, int64_t pd, int64_t ph, int64_t pw) {
  TORCH_CHECK(vol.is_contiguous() && vol.dim() == 5, "patch_gather: contiguous (B, C, D, H, W) volume");
  TORCH_CHECK(index.scalar_type() == at::kLong && index.is_contiguous(), "patch_gather: int64 (B, K) index");
  c10::cuda::CUDAGuard guard(vol.device());
  const int B = (int)vol.size(0), C = (int)vol.size(1), D = (int)vol.size(2), H = (int)vol.size(3), W = (int)vol.size(4);
  const int K = (int)index.size(1);
  if (B * K == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  auto launch = [&](auto in_tag, auto out_tag) {
    using Tin = decltype(in_tag);
    using Tout = decltype(out_tag);
    patch_gather_kernel<Tin, Tout><<<B * K, threads, 0, stream>>>(
        reinterpret_cast<const Tin*>(vol.data_ptr()), index.data_ptr<int64_t>(), reinterpret_cast<Tout*>(out.data_ptr()),
        C, D, H, W, (int)pd, (int)ph, (int)pw, K);
  };
  const bool in_f = vol.scalar_type() == at::kFloat;
  const bool out_f = out.scalar_type() == at::kFloat;
  if (in_f && out_f) launch(float{}, float{});
  else if (in_f && !out_f) launch(float{}, bf16{});
  else if (!in_f && out_f) launch(bf16{}, float{});
  else launch(bf16{}, bf16{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[b, n, :] = restore[b, n] < K ? visible[b, restore[b, n], :] : token. One warp per row, 16 B
// vectors (d % 8 == 0).
__global__ void mae_restore_fwd_kernel(const bf16* __restrict__ visible, const bf16* __restrict__ token,
                                       const int64_t* __restrict__ restore, bf16* __restrict__ out, int B, int N,
                                       int K, int d) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= B * N) return;
  const int b = row / N;
  const int64_t r = restore[row];
  const uint4* src = r < K ? reinterpret_cast<const uint4*>(visible + ((size_t)b * K + r) * d)
                           : reinterpret_cast<const uint4*>(token);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)row * d);
  for (int c = lane; c < d / 8; c += 32) dst[c] = src[c];
}

// dvis[b, restore[b, n]] = dout[b, n] for visible rows; dtoken += sum of the others. Each CTA
// reduces its masked rows in registers and shared memory, then one atomic per column.
__global__ void mae_restore_bwd_kernel(const bf16* __restrict__ dout, const int64_t* __restrict__ restore,
                                       bf16* __restrict__ dvis, float* __restrict__ dtok, int B, int N, int K, int d) {
  extern __shared__ float part[];  // [d]
  for (int i = threadIdx.x; i < d; i += blockDim.x) part[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int warps = blockDim.x / 32;
  constexpr int kMaxVec = 8;  // d <= 2048
  float acc[kMaxVec * 8];
#pragma unroll
  for (int i = 0; i < kMaxVec * 8; ++i) acc[i] = 0.f;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < B * N; row += gridDim.x * warps) {
    const int b = row / N;
    const int64_t r = restore[row];
    const uint4* src = reinterpret_cast<const uint4*>(dout + (size_t)row * d);
    if (r < K) {
      uint4* dst = reinterpret_cast<uint4*>(dvis + ((size_t)b * K + r) * d);
      for (int c = lane; c < d / 8; c += 32) dst[c] = src[c];
    } else {
#pragma unroll
      for (int vi = 0; vi < kMaxVec; ++vi) {
        const int c = lane + 32 * vi;
        if (c < d / 8) {
          uint4 u = src[c];
          uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            acc[vi * 8 + 2 * h] += bf16_lo(w[h]);
            acc[vi * 8 + 2 * h + 1] += bf16_hi(w[h]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int vi = 0; vi < kMaxVec; ++vi) {
    const int c = lane + 32 * vi;
    if (c < d / 8)
#pragma unroll
      for (int e = 0; e < 8; ++e) atomicAdd(&part[c * 8 + e], acc[vi * 8 + e]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) atomicAdd(dtok + i, part[i]);
}

void mae_restore_fwd(torch::Tensor visible, torch::Tensor token, torch::Tensor restore, torch::Tensor out) {
  TORCH_CHECK(visible.scalar_type() == at::kBFloat16 && visible.is_contiguous(), "mae_restore: bf16 visible");
  const int B = (int)restore.size(0), N = (int)restore.size(1), K = (int)visible.size(1), d = (int)visible.size(2);
  TORCH_CHECK(d % 8 == 0, "mae_restore: width must be a multiple of 8");
  c10::cuda::CUDAGuard guard(visible.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const long rows = (long)B * N;
  if (rows == 0) return;
  mae_restore_fwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const bf16*>(visible.data_ptr()), reinterpret_cast<const bf16*>(token.data_ptr()),
      restore.data_ptr<int64_t>(), reinterpret_cast<bf16*>(out.data_ptr()), B, N, K, d);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mae_restore_bwd(torch::Tensor dout, torch::Tensor restore, torch::Tensor dvis, torch::Tensor dtok) {
  const int B = (int)restore.size(0), N = (int)restore.size(1), K = (int)dvis.size(1), d = (int)dvis.size(2);
  TORCH_CHECK(d % 8 == 0 && d <= 2048, "mae_restore_bwd: width must be a multiple of 8 and at most 2048");
  c10::cuda::CUDAGuard guard(dout.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dout.get_device()));
  const int grid = std::max(1, std::min(sms, (B * N + 7) / 8));
  mae_restore_bwd_kernel<<<grid, 256, d * sizeof(float), stream>>>(
      reinterpret_cast<const bf16*>(dout.data_ptr()), restore.data_ptr<int64_t>(),
      reinterpret_cast<bf16*>(dvis.data_ptr()), dtok.data_ptr<float>(), B, N, K, d);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One CTA per (b, n) patch. The patch is read as runs of 8 voxels along W (pw % 8 == 0), so every
// load is 16 B (bf16) or 32 B (fp32). Pass 1: shifted sum and sum of squares (shift = the patch's
// first voxel, which keeps the variance well conditioned); pass 2 re-reads the runs (L1/L2 hits),
// forms the normalised target and writes the loss contribution and the gradient.
// Masked patches: target = (x - mean) / sqrt(var_unbiased + 1e-6) (or x itself);
// loss += sum((pred - target)^2) / P / count; grad = 2 (pred - target) / P / count.
// Visible patches: grad = 0. `count` = max(1, sum(mask)) is read from the device.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<bf16>(const bf16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    v[2 * h] = bf16_lo(w[h]);
    v[2 * h + 1] = bf16_hi(w[h]);
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<bf16>(bf16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                                            pack_bf16x2(v[6], v[7]));
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

template <typename TP, typename TV>
__global__ void norm_pix_mse_kernel(const TP* __restrict__ pred, const TV* __restrict__ vol,
                                    const float* __restrict__ mask, const float* __restrict__ count,
                                    float* __restrict__ loss, TP* __restrict__ grad, int C, int D, int H, int W,
                                    int pd, int ph, int pw, int N, int norm_pix) {
  const int row = blockIdx.x;
  const int b = row / N, n = row % N;
  const int vp = pd * ph * pw;
  const int P = C * vp;
  const int runs = P / 8;
  const TP* pr = pred + (size_t)row * P;
  TP* gr = grad + (size_t)row * P;
  const float mk = mask[row];
  if (mk == 0.f) {
    const float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int u = threadIdx.x; u < runs; u += blockDim.x) store8<TP>(gr + u * 8, z);
    return;
  }
  const int gh = H / ph, gw = W / pw;
  const int zd = n / (gh * gw), zh = (n / gw) % gh, zw = n % gw;
  const int runs_per_row = pw / 8;
  auto run_ptr = [&](int u) -> const TV* {
    const int e = u * 8;
    const int c = e / vp;
    int r = e % vp;
    const int a = r / (ph * pw);
    r %= ph * pw;
    const int j = r / pw, l = r % pw;
    return vol + ((((size_t)b * C + c) * D + (zd * pd + a)) * H + (zh * ph + j)) * W + (zw * pw + l);
  };
  (void)runs_per_row;
  __shared__ float red[32];
  __shared__ float shift_s;
  auto block_sum = [&](float v) -> float {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) tot += red[w];
    return tot;
  };
  float mean = 0.f, inv = 1.f;
  if (norm_pix) {
    if (threadIdx.x == 0) shift_s = to_f<TV>(*run_ptr(0));
    __syncthreads();
    const float shift = shift_s;
    float s = 0.f, ss = 0.f;
    for (int u = threadIdx.x; u < runs; u += blockDim.x) {
      float x[8];
      load8<TV>(run_ptr(u), x);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = x[j] - shift;
        s += d;
        ss += d * d;
      }
    }
    const float tot_s = block_sum(s);
    const float tot_ss = block_sum(ss);
    const float m_shifted = tot_s / P;
    mean = shift + m_shifted;
    const float var = fmaxf(tot_ss - tot_s * m_shifted, 0.f) / (float)(P > 1 ? P - 1 : 1);
    inv = rsqrtf(var + 1e-6f);
  }
  const float cnt = *count;
  const float gscale = 2.f / (float)P / cnt * mk;
  float se = 0.f;
  for (int u = threadIdx.x; u < runs; u += blockDim.x) {
    float x[8], p[8], g[8];
    load8<TV>(run_ptr(u), x);
    load8<TP>(pr + u * 8, p);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float diff = p[j] - (x[j] - mean) * inv;
      se += diff * diff;
      g[j] = diff * gscale;
    }
    store8<TP>(gr + u * 8, g);
  }
  const float tot = block_sum(se);
  if (threadIdx.x == 0) atomicAdd(loss, tot * mk / (float)P / cnt);
}

// SimMIM's loss (reference `src/algorithms/simmim.py:197-207`): per patch the mean absolute error
// between the prediction and the target patch (read straight from the volume, optionally normalised
// by its own mean and unbiased variance + 1e-6), averaged over the masked patches; the visible
// patches' mean is accumulated as a metric. One CTA per patch; the gradient sign(p - t) / P / count
// is written for masked patches (zero for visible ones) in the same pass. sums[0] += masked error,
// sums[1] += visible error (both already divided by their patch counts).
template <typename TP, typename TV>
__global__ void masked_l1_kernel(const TP* __restrict__ pred, const TV* __restrict__ vol, const float* __restrict__ mask,
                                 const float* __restrict__ counts, float* __restrict__ sums, TP* __restrict__ grad, int C,
                                 int D, int H, int W, int pd, int ph, int pw, int N, int norm_pix) {
  const int row = blockIdx.x;
  const int b = row / N, n = row % N;
  const int vp = pd * ph * pw;
  const int P = C * vp;
  const int runs = P / 8;
  const TP* pr = pred + (size_t)row * P;
  TP* gr = grad + (size_t)row * P;
  const float mk = mask[row];
  const int gh = H / ph, gw = W / pw;
  const int zd = n / (gh * gw), zh = (n / gw) % gh, zw = n % gw;
  auto run_ptr = [&](int u) -> const TV* {
    const int e = u * 8;
    const int c = e / vp;
    int r = e % vp;
    const int a = r / (ph * pw);
    r %= ph * pw;
    const int j = r / pw, l = r % pw;
    return vol + ((((size_t)b * C + c) * D + (zd * pd + a)) * H + (zh * ph + j)) * W + (zw * pw + l);
  };
  __shared__ float red[32];
  __shared__ float shift_s;
  auto block_sum = [&](float v) -> float {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) tot += red[w];
    return tot;
  };
  float mean = 0.f, inv = 1.f;
  if (norm_pix) {
    if (threadIdx.x == 0) shift_s = to_f<TV>(*run_ptr(0));
    __syncthreads();
    const float shift = shift_s;
    float s = 0.f, ss = 0.f;
    for (int u = threadIdx.x; u < runs; u += blockDim.x) {
      float x[8];
      load8<TV>(run_ptr(u), x);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = x[j] - shift;
        s += d;
        ss += d * d;
      }
    }
    const float tot_s = block_sum(s);
    const float tot_ss = block_sum(ss);
    const float m_shifted = tot_s / P;
    mean = shift + m_shifted;
    const float var = fmaxf(tot_ss - tot_s * m_shifted, 0.f) / (float)(P > 1 ? P - 1 : 1);
    inv = rsqrtf(var + 1e-6f);
  }
  const float n_masked = counts[0], n_visible = counts[1];
  const float gscale = mk != 0.f ? 1.f / (float)P / n_masked : 0.f;
  float ae = 0.f;
  for (int u = threadIdx.x; u < runs; u += blockDim.x) {
    float x[8], p[8], g[8];
    load8<TV>(run_ptr(u), x);
    load8<TP>(pr + u * 8, p);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float diff = p[j] - (x[j] - mean) * inv;
      ae += fabsf(diff);
      g[j] = diff > 0.f ? gscale : (diff < 0.f ? -gscale : 0.f);
    }
    store8<TP>(gr + u * 8, g);
  }
  const float tot = block_sum(ae) / (float)P;
  if (threadIdx.x == 0) {
    if (mk != 0.f) atomicAdd(&sums[0], tot / n_masked);
    else atomicAdd(&sums[1], tot / n_visible);
  }
}

void masked_l1(torch::Tensor pred, torch::Tensor vol, torch::Tensor mask, torch::Tensor sums, torch::Tensor grad,
               int64_t pd, int64_t ph, int64_t pw, bool norm_pix) {
  TORCH_CHECK(pred.is_cuda() && pred.is_contiguous() && vol.is_contiguous() && mask.is_contiguous(),
              "masked_l1: contiguous CUDA inputs");
  TORCH_CHECK(mask.scalar_type() == at::kFloat && sums.scalar_type() == at::kFloat && sums.numel() == 2,
              "masked_l1: fp32 mask and a 2-element fp32 sums buffer");
  const int B = (int)vol.size(0), C = (int)vol.size(1), D = (int)vol.size(2), H = (int)vol.size(3), W = (int)vol.size(4);
  const int N = (int)pred.size(1);
  const int P = (int)pred.size(2);
  TORCH_CHECK(P == C * pd * ph * pw, "masked_l1: patch width mismatch");
  TORCH_CHECK(pw % 8 == 0 && W % 8 == 0, "masked_l1: the W extent of a patch must be a multiple of 8");
  TORCH_CHECK(mask.numel() == (int64_t)B * N, "masked_l1: one mask value per patch");
  c10::cuda::CUDAGuard guard(pred.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto masked = mask.sum();
  auto counts = torch::stack({masked.clamp_min(1.0), (masked.neg() + (double)mask.numel()).clamp_min(1.0)});
  C10_CUDA_CHECK(cudaMemsetAsync(sums.data_ptr(), 0, 2 * sizeof(float), stream));
  auto launch = [&](auto p_tag, auto v_tag) {
    using TP = decltype(p_tag);
    using TV = decltype(v_tag);
    masked_l1_kernel<TP, TV><<<B * N, 256, 0, stream>>>(
        reinterpret_cast<const TP*>(pred.data_ptr()), reinterpret_cast<const TV*>(vol.data_ptr()), mask.data_ptr<float>(),
        counts.data_ptr<float>(), sums.data_ptr<float>(), reinterpret_cast<TP*>(grad.data_ptr()), C, D, H, W, (int)pd,
        (int)ph, (int)pw, N, norm_pix ? 1 : 0);
  };
  const bool pf = pred.scalar_type() == at::kFloat, vf = vol.scalar_type() == at::kFloat;
  if (pf && vf) launch(float{}, float{});
  else if (pf && !vf) launch(float{}, bf16{});
  else if (!pf && vf) launch(bf16{}, float{});
  else launch(bf16{}, bf16{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void norm_pix_mse(torch::Tensor pred, torch::Tensor vol, torch::Tensor mask, torch::Tensor loss, torch::Tensor grad,
                  int64_t pd, int64_t ph, int64_t pw, bool norm_pix) {
  TORCH_CHECK(pred.is_contiguous() && vol.is_contiguous() && mask.is_contiguous(), "norm_pix_mse: contiguous inputs");
  const int B = (int)vol.size(0), C = (int)vol.size(1), D = (int)vol.size(2), H = (int)vol.size(3), W = (int)vol.size(4);
  const int N = (int)pred.size(1);
  const int P = (int)pred.size(2);
  TORCH_CHECK(P == C * pd * ph * pw, "norm_pix_mse: patch width mismatch");
  TORCH_CHECK(pw % 8 == 0 && W % 8 == 0, "norm_pix_mse: the W extent of a patch must be a multiple of 8");
  c10::cuda::CUDAGuard guard(pred.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto count = mask.sum().clamp_min(1.0);
  C10_CUDA_CHECK(cudaMemsetAsync(loss.data_ptr(), 0, sizeof(float), stream));
  auto launch = [&](auto p_tag, auto v_tag) {
    using TP = decltype(p_tag);
    using TV = decltype(v_tag);
    norm_pix_mse_kernel<TP, TV><<<B * N, 256, 0, stream>>>(
        reinterpret_cast<const TP*>(pred.data_ptr()), reinterpret_cast<const TV*>(vol.data_ptr()), mask.data_ptr<float>(),
        count.data_ptr<float>(), loss.data_ptr<float>(), reinterpret_cast<TP*>(grad.data_ptr()), C, D, H, W, (int)pd,
        (int)ph, (int)pw, N, norm_pix ? 1 : 0);
  };
  const bool pf = pred.scalar_type() == at::kFloat, vf = vol.scalar_type() == at::kFloat;
  if (pf && vf) launch(float{}, float{});
  else if (pf && !vf) launch(float{}, bf16{});
  else if (!pf && vf) launch(bf16{}, float{});
  else launch(bf16{}, bf16{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
