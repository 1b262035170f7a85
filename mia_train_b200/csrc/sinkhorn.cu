// Sinkhorn-Knopp centring of teacher logits (DINO / iBOT) as scaling vectors.
//
// With E[b, k] = exp(x[b, k] / T), every iterate of the reference's loop (normalise by the global
// sum, then alternately by the all-reduced prototype sums / K and the per-sample sums / B) has the
// form Q[b, k] = E[b, k] * r[k] * s[b]. Each iteration therefore needs only two reductions over E:
// per-prototype sums A[k] = sum_b E[b, k] s[b] (all-reduced across ranks by the caller) and
// per-sample sums T[b] = sum_k E[b, k] r[k]; the matrix is written once at the end. E is recomputed
// from the logits in every pass (bf16 or fp32 input, 8 columns per thread), so nothing of size
// B x K is stored between passes.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mia {
namespace {

constexpr int kSkThreads = 256;
constexpr int kSkCols = 8;  // columns per thread

__device__ __forceinline__ float sk_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16_lo(w[i]);
    v[2 * i + 1] = bf16_hi(w[i]);
  }
}

// A[k] += sum over this CTA's rows b of exp(x[b, k] / T) * s[b] (s == nullptr: 1).
template <typename T>
__global__ void __launch_bounds__(kSkThreads) sk_colsum_kernel(const T* __restrict__ x, int B, int K, float scale_log2,
                                                               const float* __restrict__ s, int rows_per_cta,
                                                               float* __restrict__ out) {
  const int k0 = (blockIdx.x * kSkThreads + threadIdx.x) * kSkCols;
  if (k0 >= K) return;
  const int b0 = blockIdx.y * rows_per_cta;
  const int b1 = min(B, b0 + rows_per_cta);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int b = b0; b < b1; ++b) {
    float v[8];
    load8<T>(x + (size_t)b * K + k0, v);
    const float sb = s != nullptr ? s[b] : 1.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += sk_exp2(v[j] * scale_log2) * sb;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) atomicAdd(out + k0 + j, acc[j]);
}

// T[b] += sum over this CTA's columns k of exp(x[b, k] / T) * r[k].
template <typename T>
__global__ void __launch_bounds__(kSkThreads) sk_rowsum_kernel(const T* __restrict__ x, int K, float scale_log2,
                                                               const float* __restrict__ r, int cols_per_cta,
                                                               float* __restrict__ out) {
  const int b = blockIdx.y;
  const int c0 = blockIdx.x * cols_per_cta;
  const int c1 = min(K, c0 + cols_per_cta);
  const T* row = x + (size_t)b * K;
  float acc = 0.f;
  for (int k = c0 + threadIdx.x * kSkCols; k < c1; k += kSkThreads * kSkCols) {
    float v[8], rr[8];
    load8<T>(row + k, v);
    load8<float>(r + k, rr);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += sk_exp2(v[j] * scale_log2) * rr[j];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ float ws[kSkThreads / 32];
  if (threadIdx.x % 32 == 0) ws[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kSkThreads / 32; ++w) t += ws[w];
    atomicAdd(out + b, t);
  }
}

// P[b, k] = exp(x[b, k] / T) * r[k] * s[b] * factor (fp32 output).
template <typename T>
__global__ void __launch_bounds__(kSkThreads) sk_scale_kernel(const T* __restrict__ x, int B, int K, float scale_log2,
                                                              const float* __restrict__ r, const float* __restrict__ s,
                                                              float factor, float* __restrict__ out) {
  const size_t total = (size_t)B * K / kSkCols;
  for (size_t i = (size_t)blockIdx.x * kSkThreads + threadIdx.x; i < total; i += (size_t)gridDim.x * kSkThreads) {
    const size_t e = i * kSkCols;
    const int b = (int)(e / K), k = (int)(e % K);
    float v[8], rr[8];
    load8<T>(x + e, v);
    load8<float>(r + k, rr);
    const float sb = s[b] * factor;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = sk_exp2(v[j] * scale_log2) * rr[j] * sb;
    *reinterpret_cast<float4*>(out + e) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(out + e + 4) = make_float4(o[4], o[5], o[6], o[7]);
  }
}

int sm_count(const torch::Tensor& t) {
  int v = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, t.get_device()));
  return v;
}

void check_logits(const torch::Tensor& x, const char* who) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() &&
                  (x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16),
              who, ": contiguous (B, K) fp32 / bf16 CUDA logits");
  TORCH_CHECK(x.size(1) % kSkCols == 0, who, ": K must be a multiple of 8");
}

constexpr float kLog2eF = 1.4426950408889634f;

}  // namespace

// out (K,) fp32, zeroed here: sum_b exp(x[b, k] / T) * s[b] (s optional).
void sinkhorn_colsum(torch::Tensor x, double temperature, c10::optional<torch::Tensor> s, torch::Tensor out) {
  check_logits(x, "sinkhorn_colsum");
  const int B = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == K, "sinkhorn_colsum: (K,) fp32 out");
  TORCH_CHECK(!s.has_value() || (s->scalar_type() == at::kFloat && s->is_contiguous() && s->numel() == B),
              "sinkhorn_colsum: (B,) fp32 s");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemsetAsync(out.data_ptr(), 0, (size_t)K * 4, stream));
  if (B == 0 || K == 0) return;
  const int gx = (K / kSkCols + kSkThreads - 1) / kSkThreads;
  const int gy = std::max(1, std::min(B, (4 * sm_count(x) + gx - 1) / gx));
  const int rows = (B + gy - 1) / gy;
  const float sl = (float)(kLog2eF / temperature);
  const float* sp = s.has_value() ? s->data_ptr<float>() : nullptr;
  if (x.scalar_type() == at::kFloat)
    sk_colsum_kernel<float><<<dim3(gx, gy), kSkThreads, 0, stream>>>(x.data_ptr<float>(), B, K, sl, sp, rows,
                                                                     out.data_ptr<float>());
  else
    sk_colsum_kernel<__nv_bfloat16><<<dim3(gx, gy), kSkThreads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), B, K, sl, sp, rows, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out (B,) fp32, zeroed here: sum_k exp(x[b, k] / T) * r[k].
void sinkhorn_rowsum(torch::Tensor x, double temperature, torch::Tensor r, torch::Tensor out) {
  check_logits(x, "sinkhorn_rowsum");
  const int B = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(r.scalar_type() == at::kFloat && r.is_contiguous() && r.numel() == K, "sinkhorn_rowsum: (K,) fp32 r");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == B, "sinkhorn_rowsum: (B,) fp32 out");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemsetAsync(out.data_ptr(), 0, (size_t)B * 4, stream));
  if (B == 0 || K == 0) return;
  const int per_iter = kSkThreads * kSkCols;
  const int gx_max = (K + per_iter - 1) / per_iter;
  const int gx = std::max(1, std::min(gx_max, (4 * sm_count(x) + B - 1) / B));
  const int cols = ((K + gx - 1) / gx + kSkCols - 1) / kSkCols * kSkCols;
  const float sl = (float)(kLog2eF / temperature);
  if (x.scalar_type() == at::kFloat)
    sk_rowsum_kernel<float><<<dim3(gx, B), kSkThreads, 0, stream>>>(x.data_ptr<float>(), K, sl, r.data_ptr<float>(),
                                                                    cols, out.data_ptr<float>());
  else
    sk_rowsum_kernel<__nv_bfloat16><<<dim3(gx, B), kSkThreads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), K, sl, r.data_ptr<float>(), cols, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out (B, K) fp32 = exp(x / T) * r[k] * s[b] * factor.
void sinkhorn_scale(torch::Tensor x, double temperature, torch::Tensor r, torch::Tensor s, double factor,
                    torch::Tensor out) {
  check_logits(x, "sinkhorn_scale");
  const int B = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(r.scalar_type() == at::kFloat && r.is_contiguous() && r.numel() == K, "sinkhorn_scale: (K,) fp32 r");
  TORCH_CHECK(s.scalar_type() == at::kFloat && s.is_contiguous() && s.numel() == B, "sinkhorn_scale: (B,) fp32 s");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.sizes() == x.sizes(),
              "sinkhorn_scale: (B, K) fp32 out");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (B == 0 || K == 0) return;
  const size_t work = (size_t)B * K / kSkCols;
  const int grid =
      (int)std::max<size_t>(1, std::min<size_t>((work + kSkThreads - 1) / kSkThreads, 8 * (size_t)sm_count(x)));
  const float sl = (float)(kLog2eF / temperature);
  if (x.scalar_type() == at::kFloat)
    sk_scale_kernel<float><<<grid, kSkThreads, 0, stream>>>(x.data_ptr<float>(), B, K, sl, r.data_ptr<float>(),
                                                            s.data_ptr<float>(), (float)factor, out.data_ptr<float>());
  else
    sk_scale_kernel<__nv_bfloat16><<<grid, kSkThreads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), B, K, sl, r.data_ptr<float>(), s.data_ptr<float>(),
        (float)factor, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
