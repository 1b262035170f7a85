// LayerNorm / RMSNorm forward and backward, one warp per row, fp32 statistics.
//
// Forward writes y (input dtype), the row mean (0 for RMSNorm) and 1/sqrt(var + eps). Backward
// recomputes xhat from them:
//   g   = dy * w
//   dx  = rstd * (g - mean(g) - xhat * mean(g * xhat))        (LayerNorm)
//   dx  = rstd * (g - xhat * mean(g * xhat))                  (RMSNorm)
//   dw += sum_rows dy * xhat,   db += sum_rows dy
// Backward runs as two kernels: dX with one warp per row, and the weight/bias gradients as a column
// reduction over row slabs (one atomic per column per CTA, about one CTA per SM).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <type_traits>

#include "common.cuh"

namespace mia {

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      v[2 * h] = bf16_lo(w[h]);
      v[2 * h + 1] = bf16_hi(w[h]);
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                              pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Row held in registers (n == NCH * 256: eight elements per lane per 256-column chunk), read once;
// mean and variance from the registers (two-pass in registers, so no catastrophic cancellation).
template <typename T, int NCH>
__global__ void layernorm_fwd_reg_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                         const float* __restrict__ b, T* __restrict__ y, float* __restrict__ mean_out,
                                         float* __restrict__ rstd_out, int rows, float eps, int rms) {
  constexpr int n = NCH * 256;
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const T* xr = x + (size_t)row * n;
    float v[NCH][8];
#pragma unroll
    for (int c = 0; c < NCH; ++c) Vec8<T>::load(xr + c * 256 + lane * 8, v[c]);
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[c][j];
    const float mean = rms ? 0.f : warp_sum(s) * (1.0f / n);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[c][j] - mean;
        ss += d * d;
      }
    const float rstd = rsqrtf(warp_sum(ss) * (1.0f / n) + eps);
    T* yr = y + (size_t)row * n;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      float wv[8], bv[8];
      if (w != nullptr) {
        Vec8<float>::load(w + col, wv);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) wv[j] = 1.f;
      }
      if (b != nullptr) {
        Vec8<float>::load(b + col, bv);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) bv[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[c][j] = (v[c][j] - mean) * rstd * wv[j] + bv[j];
      Vec8<T>::store(yr + col, v[c]);
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

template <typename T>
__global__ void layernorm_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                                     T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                     int rows, int n, float eps, int rms) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const T* xr = x + (size_t)row * n;
    float s = 0.f;
    for (int c = lane * 8; c < n; c += 256) {
      float v[8];
      Vec8<T>::load(xr + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[j];
    }
    const float mean = rms ? 0.f : warp_sum(s) / n;
    float ss = 0.f;
    for (int c = lane * 8; c < n; c += 256) {
      float v[8];
      Vec8<T>::load(xr + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[j] - mean;
        ss += d * d;
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / n + eps);
    T* yr = y + (size_t)row * n;
    for (int c = lane * 8; c < n; c += 256) {
      float v[8];
      Vec8<T>::load(xr + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float o = (v[j] - mean) * rstd;
        if (w != nullptr) o *= __ldg(w + c + j);
        if (b != nullptr) o += __ldg(b + c + j);
        v[j] = o;
      }
      Vec8<T>::store(yr + c, v);
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

// dX: one warp per row, the row held in registers (NCH chunks of 8 columns per lane). `dres`, when
// given, is the gradient that reaches x through a residual branch; it is added to dX here, which
// saves autograd's separate sum of the two gradients.
template <typename T, int NCH>
__global__ void layernorm_bwd_dx_kernel(const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
                                        const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                                        T* __restrict__ dx, int rows, int n, int rms, const T* __restrict__ dres) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const T* xr = x + (size_t)row * n;
    const T* gr = dy + (size_t)row * n;
    const float mean = mean_in[row];
    const float rstd = rstd_in[row];
    float xh[NCH][8], g[NCH][8];
    float sum_g = 0.f, sum_gx = 0.f;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c = lane * 8 + ch * 256;
      if (c < n) {
        float xv[8], gv[8];
        Vec8<T>::load(xr + c, xv);
        Vec8<T>::load(gr + c, gv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[ch][j] = (xv[j] - mean) * rstd;
          g[ch][j] = gv[j] * (w != nullptr ? __ldg(w + c + j) : 1.f);
          sum_g += g[ch][j];
          sum_gx += g[ch][j] * xh[ch][j];
        }
      }
    }
    const float mg = rms ? 0.f : warp_sum(sum_g) / n;
    const float mgx = warp_sum(sum_gx) / n;
    T* dr = dx + (size_t)row * n;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c = lane * 8 + ch * 256;
      if (c < n) {
        float o[8], rg[8];
        if (dres != nullptr) {
          Vec8<T>::load(dres + (size_t)row * n + c, rg);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) rg[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rstd * (g[ch][j] - mg - xh[ch][j] * mgx) + rg[j];
        Vec8<T>::store(dr + c, o);
      }
    }
  }
}

// dw[c] += sum_r dy[r, c] * xhat[r, c], db[c] += sum_r dy[r, c]. A CTA owns 256 columns (8 per lane)
// and a slab of rows split over its 8 warps; warps are combined in shared memory and the CTA adds one
// value per column (the slab height keeps the CTA count near the SM count).
template <typename T>
__global__ void __launch_bounds__(256) layernorm_bwd_param_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                                  const float* __restrict__ mean_in,
                                                                  const float* __restrict__ rstd_in,
                                                                  float* __restrict__ dw, float* __restrict__ db,
                                                                  int rows, int n, int rows_per_cta) {
  __shared__ float part[2][8][256];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c = blockIdx.x * 256 + lane * 8;
  const int r_begin = blockIdx.y * rows_per_cta;
  const int r_end = min(rows, r_begin + rows_per_cta);
  float aw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, ab[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c < n) {
    // 4 rows per warp per iteration: their 8 vector loads are all in flight before the math.
    for (int r = r_begin + warp; r < r_end; r += 32) {
      float xv[4][8], gv[4][8], mean[4], rstd[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r + 8 * u;
        if (rr < r_end) {
          Vec8<T>::load(x + (size_t)rr * n + c, xv[u]);
          Vec8<T>::load(dy + (size_t)rr * n + c, gv[u]);
          mean[u] = mean_in[rr];
          rstd[u] = rstd_in[rr];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[u][j] = gv[u][j] = 0.f;
          mean[u] = rstd[u] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          aw[j] += gv[u][j] * (xv[u][j] - mean[u]) * rstd[u];
          ab[j] += gv[u][j];
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    part[0][warp][lane * 8 + j] = aw[j];
    part[1][warp][lane * 8 + j] = ab[j];
  }
  __syncthreads();
  const int col = blockIdx.x * 256 + threadIdx.x;
  if (col < n) {
    float sw = 0.f, sb = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      sw += part[0][k][threadIdx.x];
      sb += part[1][k][threadIdx.x];
    }
    if (dw != nullptr) atomicAdd(dw + col, sw);
    if (db != nullptr) atomicAdd(db + col, sb);
  }
}

static int sm_count(const torch::Tensor& t) {
  int v = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, t.get_device()));
  return v;
}

void layernorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> w, c10::optional<torch::Tensor> b, torch::Tensor y,
                   torch::Tensor mean, torch::Tensor rstd, double eps, bool rms) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 2, "layernorm_fwd: contiguous 2-D CUDA input");
  const int rows = (int)x.size(0), n = (int)x.size(1);
  TORCH_CHECK(n % 8 == 0, "layernorm: hidden size must be a multiple of 8");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  const float* bp = b.has_value() ? b->data_ptr<float>() : nullptr;
  if (rows == 0) return;
  const int threads = 256;
  const int grid = std::min((rows + 7) / 8, sm_count(x) * 8);
  if (n % 256 == 0 && n / 256 <= 8) {
    auto launch = [&](auto tag, auto nch) {
      using T = decltype(tag);
      constexpr int NCH = decltype(nch)::value;
      layernorm_fwd_reg_kernel<T, NCH><<<grid, threads, 0, stream>>>(
          reinterpret_cast<const T*>(x.data_ptr()), wp, bp, reinterpret_cast<T*>(y.data_ptr()),
          mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, (float)eps, rms ? 1 : 0);
    };
    auto by_width = [&](auto tag) {
      switch (n / 256) {
        case 1: launch(tag, std::integral_constant<int, 1>{}); break;
        case 2: launch(tag, std::integral_constant<int, 2>{}); break;
        case 3: launch(tag, std::integral_constant<int, 3>{}); break;
        case 4: launch(tag, std::integral_constant<int, 4>{}); break;
        case 5: launch(tag, std::integral_constant<int, 5>{}); break;
        case 6: launch(tag, std::integral_constant<int, 6>{}); break;
        case 7: launch(tag, std::integral_constant<int, 7>{}); break;
        default: launch(tag, std::integral_constant<int, 8>{}); break;
      }
    };
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "layernorm: bf16 or fp32 input");
    if (x.scalar_type() == at::kBFloat16) by_width(__nv_bfloat16{});
    else by_width(float{});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (x.scalar_type() == at::kBFloat16) {
    layernorm_fwd_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), wp, bp, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
        mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, n, (float)eps, rms ? 1 : 0);
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "layernorm: bf16 or fp32 input");
    layernorm_fwd_kernel<float><<<grid, threads, 0, stream>>>(x.data_ptr<float>(), wp, bp, y.data_ptr<float>(),
                                                              mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, n,
                                                              (float)eps, rms ? 1 : 0);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void layernorm_bwd(torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> w, torch::Tensor mean,
                   torch::Tensor rstd, torch::Tensor dx, c10::optional<torch::Tensor> dw,
                   c10::optional<torch::Tensor> db, bool rms, c10::optional<torch::Tensor> dres) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.sizes() == x.sizes(), "layernorm_bwd: shapes");
  TORCH_CHECK(!dres.has_value() || (dres->is_contiguous() && dres->sizes() == x.sizes() &&
                                    dres->scalar_type() == x.scalar_type()),
              "layernorm_bwd: residual gradient must match x");
  const int rows = (int)x.size(0), n = (int)x.size(1);
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return;
  TORCH_CHECK(n <= 256 * 8, "layernorm_bwd: hidden size above 2048 is not supported");
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  float* dwp = dw.has_value() ? dw->data_ptr<float>() : nullptr;
  float* dbp = db.has_value() ? db->data_ptr<float>() : nullptr;
  const int sms = sm_count(x);
  const int dx_grid = std::max(1, std::min(8 * sms, (rows + 7) / 8));
  const int gx = (n + 255) / 256;
  const int gy = std::max(1, std::min((rows + 31) / 32, (sms + gx - 1) / gx));
  const int rows_per_cta = (rows + gy - 1) / gy;
  auto run = [&](auto tag, auto nch) {
    using T = decltype(tag);
    constexpr int NCH = decltype(nch)::value;
    layernorm_bwd_dx_kernel<T, NCH><<<dx_grid, 256, 0, stream>>>(
        reinterpret_cast<const T*>(dy.data_ptr()), reinterpret_cast<const T*>(x.data_ptr()), wp, mean.data_ptr<float>(),
        rstd.data_ptr<float>(), reinterpret_cast<T*>(dx.data_ptr()), rows, n, rms ? 1 : 0,
        dres.has_value() ? reinterpret_cast<const T*>(dres->data_ptr()) : nullptr);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    if (dwp != nullptr || dbp != nullptr) {
      layernorm_bwd_param_kernel<T><<<dim3(gx, gy), 256, 0, stream>>>(
          reinterpret_cast<const T*>(dy.data_ptr()), reinterpret_cast<const T*>(x.data_ptr()), mean.data_ptr<float>(),
          rstd.data_ptr<float>(), dwp, dbp, rows, n, rows_per_cta);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
    }
  };
  auto by_width = [&](auto tag) {
    if (n <= 256) run(tag, std::integral_constant<int, 1>{});
    else if (n <= 512) run(tag, std::integral_constant<int, 2>{});
    else if (n <= 1024) run(tag, std::integral_constant<int, 4>{});
    else run(tag, std::integral_constant<int, 8>{});
  };
  if (x.scalar_type() == at::kBFloat16) by_width(__nv_bfloat16{});
  else by_width(float{});
}

}  // namespace mia
