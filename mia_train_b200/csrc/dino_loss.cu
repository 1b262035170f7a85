// Soft-target cross-entropy of the DINO and iBOT objectives over the prototype axis, and KoLeo.
//
//   loss_i = sum_j w_ij * ( lse_i * T1_j - <T_j, S_i> / tau ),   lse_i = logsumexp_k(S_ik / tau)
//
// S (R, K) are student logits (bf16 or fp32), T (Rt, K) teacher probabilities (fp32), T1_j =
// sum_k T_jk, and each student row i is paired with up to `n_pairs` teacher rows tidx[i, j] with
// weights w[i, j] (a weight of 0 skips the pair: the DINO loss ignores same-view pairs that way;
// iBOT pairs each masked patch with its own teacher row and its per-sample weight). This is
// -sum_j w_ij sum_k T_jk log softmax(S_i / tau)_k, written so one pass over a student row gives the
// log-sum-exp (online max / sum) and the pair dot products together. The reference materialises
// log_softmax in fp32 and reduces it with einsum (`src/algorithms/dinov3/losses.py:75-173`).
//
// Backward, with g the upstream gradient of sum_i loss_i:
//   dS_ik = g / tau * ( c1_i softmax(S_i / tau)_k - sum_j w_ij T_jk ),  c1_i = sum_j w_ij T1_j.
//
// One CTA per student row; 8 consecutive elements per thread and load (16 bytes of bf16).
//
// KoLeo: for L2-normalised rows x_i (B <= 1024, one CTA), the nearest neighbour n(i) by dot
// product (self excluded), d_i = || x_i - x_n(i) + eps ||, loss = -mean_i log(d_i + eps), and the
// gradient through the distance and the normalisation (the neighbour choice is piecewise constant).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mia {
namespace {

constexpr int kCeThreads = 256;
constexpr int kMaxPairs = 4;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    v[2 * h] = bf16_lo(w[h]);
    v[2 * h + 1] = bf16_hi(w[h]);
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void load8_f32(const float* p, float (&v)[8]) { load8<float>(p, v); }

// Block-wide reduction of `n` values per thread (sum), result broadcast to every thread.
template <int N>
__device__ __forceinline__ void block_sum(float (&v)[N], float* scratch /* [32 * N] */) {
#pragma unroll
  for (int j = 0; j < N; ++j)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < N; ++j) scratch[warp * N + j] = v[j];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += scratch[w * N + j];
    v[j] = t;
  }
}

template <typename TS>
__global__ void __launch_bounds__(kCeThreads) soft_ce_fwd_kernel(const TS* __restrict__ S, const float* __restrict__ T,
                                                                 const int* __restrict__ tidx,
                                                                 const float* __restrict__ w, int n_pairs, int K,
                                                                 float inv_tau, float* __restrict__ lse_out,
                                                                 float* __restrict__ loss_out) {
  __shared__ float scratch[32 * (kMaxPairs + 2)];
  __shared__ float stat[2];
  const int i = blockIdx.x;
  const TS* s = S + (int64_t)i * K;
  // pass 1: max of the row
  float m = -INFINITY;
  for (int k = threadIdx.x * 8; k < K; k += kCeThreads * 8) {
    float v[8];
    load8<TS>(s + k, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) m = fmaxf(m, v[q]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (threadIdx.x % 32 == 0) scratch[threadIdx.x / 32] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = -INFINITY;
    for (int q = 0; q < kCeThreads / 32; ++q) mm = fmaxf(mm, scratch[q]);
    stat[0] = mm;
  }
  __syncthreads();
  const float mx = stat[0] * inv_tau;
  // pass 2 (the row is in L2 now): sum of exp, pair dots, teacher masses
  float acc[kMaxPairs + 1];
  float tsum[kMaxPairs];
#pragma unroll
  for (int j = 0; j <= kMaxPairs; ++j) acc[j] = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) tsum[j] = 0.f;
  for (int k = threadIdx.x * 8; k < K; k += kCeThreads * 8) {
    float v[8];
    load8<TS>(s + k, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[kMaxPairs] += __expf(v[q] * inv_tau - mx);
#pragma unroll
    for (int j = 0; j < kMaxPairs; ++j) {
      if (j < n_pairs && w[i * n_pairs + j] != 0.f) {
        float t[8];
        load8_f32(T + (int64_t)tidx[i * n_pairs + j] * K + k, t);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          acc[j] += t[q] * v[q];
          tsum[j] += t[q];
        }
      }
    }
  }
  float red[2 * kMaxPairs + 1];
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) {
    red[j] = acc[j];
    red[kMaxPairs + j] = tsum[j];
  }
  red[2 * kMaxPairs] = acc[kMaxPairs];
  __shared__ float big[32 * (2 * kMaxPairs + 1)];
  block_sum<2 * kMaxPairs + 1>(red, big);
  if (threadIdx.x == 0) {
    const float lse = mx + __logf(red[2 * kMaxPairs]);
    float loss = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPairs; ++j) {
      const float wj = j < n_pairs ? w[i * n_pairs + j] : 0.f;
      if (wj != 0.f) loss += wj * (lse * red[kMaxPairs + j] - red[j] * inv_tau);
    }
    lse_out[i] = lse;
    loss_out[i] = loss;
  }
}

template <typename TS>
__global__ void __launch_bounds__(kCeThreads) soft_ce_bwd_kernel(const TS* __restrict__ S, const float* __restrict__ T,
                                                                 const int* __restrict__ tidx,
                                                                 const float* __restrict__ w, int n_pairs, int K,
                                                                 float inv_tau, const float* __restrict__ lse,
                                                                 const float* __restrict__ grad_scale,
                                                                 TS* __restrict__ dS) {
  __shared__ float scratch[32 * kMaxPairs];
  const int i = blockIdx.x;
  const TS* s = S + (int64_t)i * K;
  // c1 = sum_j w_ij T1_j (teacher masses of the row's pairs)
  float mass[kMaxPairs];
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) mass[j] = 0.f;
  for (int k = threadIdx.x * 8; k < K; k += kCeThreads * 8) {
#pragma unroll
    for (int j = 0; j < kMaxPairs; ++j) {
      if (j < n_pairs && w[i * n_pairs + j] != 0.f) {
        float t[8];
        load8_f32(T + (int64_t)tidx[i * n_pairs + j] * K + k, t);
#pragma unroll
        for (int q = 0; q < 8; ++q) mass[j] += t[q];
      }
    }
  }
  block_sum<kMaxPairs>(mass, scratch);
  float c1 = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j)
    if (j < n_pairs) c1 += w[i * n_pairs + j] * mass[j];
  const float g = grad_scale[0] * inv_tau;
  const float l = lse[i];
  for (int k = threadIdx.x * 8; k < K; k += kCeThreads * 8) {
    float v[8], c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    load8<TS>(s + k, v);
#pragma unroll
    for (int j = 0; j < kMaxPairs; ++j) {
      if (j < n_pairs && w[i * n_pairs + j] != 0.f) {
        const float wj = w[i * n_pairs + j];
        float t[8];
        load8_f32(T + (int64_t)tidx[i * n_pairs + j] * K + k, t);
#pragma unroll
        for (int q = 0; q < 8; ++q) c[q] += wj * t[q];
      }
    }
    float d[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) d[q] = g * (c1 * __expf(v[q] * inv_tau - l) - c[q]);
    if constexpr (std::is_same<TS, float>::value) {
      float4* o = reinterpret_cast<float4*>(dS + (int64_t)i * K + k);
      o[0] = make_float4(d[0], d[1], d[2], d[3]);
      o[1] = make_float4(d[4], d[5], d[6], d[7]);
    } else {
      *reinterpret_cast<uint4*>(dS + (int64_t)i * K + k) =
          make_uint4(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]), pack_bf16x2(d[4], d[5]), pack_bf16x2(d[6], d[7]));
    }
  }
}

// ---------------------------------------------------------------------------------------- KoLeo
constexpr int kKoleoThreads = 1024;

// x (B, D) fp32 rows. xn = x / max(||x||, eps). nn[i] = argmax_{j != i} <xn_i, xn_j> (lowest index
// on ties, as argmax). dist[i] = || xn_i - xn_nn + eps ||. loss = -mean log(dist + eps).
__global__ void __launch_bounds__(kKoleoThreads) koleo_fwd_kernel(const float* __restrict__ x, int B, int D, float eps,
                                                                  float* __restrict__ xn, int* __restrict__ nn,
                                                                  float* __restrict__ dist, float* __restrict__ loss) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, warps = blockDim.x / 32;
  for (int i = warp; i < B; i += warps) {
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) ss += x[(int64_t)i * D + d] * x[(int64_t)i * D + d];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float nrm = fmaxf(sqrtf(ss), eps);
    for (int d = lane; d < D; d += 32) xn[(int64_t)i * D + d] = x[(int64_t)i * D + d] / nrm;
  }
  __syncthreads();
  for (int i = warp; i < B; i += warps) {
    float best = -INFINITY;
    int arg = 0;
    for (int j = 0; j < B; ++j) {
      float dot = 0.f;
      if (j != i) {
        for (int d = lane; d < D; d += 32) dot += xn[(int64_t)i * D + d] * xn[(int64_t)j * D + d];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      } else {
        dot = -1.f;  // the reference fills the diagonal with -1 before its argmax
      }
      if (dot > best) {
        best = dot;
        arg = j;
      }
    }
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float diff = xn[(int64_t)i * D + d] - xn[(int64_t)arg * D + d] + eps;
      ss += diff * diff;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) {
      nn[i] = arg;
      dist[i] = sqrtf(ss);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < B; ++i) t += __logf(dist[i] + eps);
    loss[0] = -t / (float)B;
  }
}

// dxn_i += coef_i (xn_i - xn_nn + eps) / dist_i ; dxn_nn -= the same ; coef_i = -g / (B (dist_i + eps));
// dx = (dxn - xn <xn, dxn>) / norm (norm clamped at eps: then the projection term is absent).
__global__ void __launch_bounds__(kKoleoThreads) koleo_bwd_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ xn,
                                                                  const int* __restrict__ nn,
                                                                  const float* __restrict__ dist, int B, int D,
                                                                  float eps, const float* __restrict__ grad,
                                                                  float* __restrict__ dxn, float* __restrict__ dx) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, warps = blockDim.x / 32;
  const float g = grad[0];
  for (int e = threadIdx.x; e < B * D; e += blockDim.x) dxn[e] = 0.f;
  __syncthreads();
  for (int i = warp; i < B; i += warps) {
    const int n = nn[i];
    const float di = fmaxf(dist[i], 1e-30f);
    const float coef = -g / ((float)B * (dist[i] + eps)) / di;
    for (int d = lane; d < D; d += 32) {
      const float diff = xn[(int64_t)i * D + d] - xn[(int64_t)n * D + d] + eps;
      atomicAdd(&dxn[(int64_t)i * D + d], coef * diff);
      atomicAdd(&dxn[(int64_t)n * D + d], -coef * diff);
    }
  }
  __syncthreads();
  for (int i = warp; i < B; i += warps) {
    float ss = 0.f, dot = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float v = x[(int64_t)i * D + d];
      ss += v * v;
      dot += xn[(int64_t)i * D + d] * dxn[(int64_t)i * D + d];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      dot += __shfl_xor_sync(0xffffffffu, dot, o);
    }
    const float nrm = sqrtf(ss);
    const bool clamped = nrm < eps;
    const float inv = 1.f / fmaxf(nrm, eps);
    for (int d = lane; d < D; d += 32) {
      const float gd = dxn[(int64_t)i * D + d];
      dx[(int64_t)i * D + d] = clamped ? gd * inv : (gd - xn[(int64_t)i * D + d] * dot) * inv;
    }
  }
}

void check_ce(const at::Tensor& S, const at::Tensor& T, const at::Tensor& tidx, const at::Tensor& w) {
  TORCH_CHECK(S.is_cuda() && S.dim() == 2 && S.is_contiguous() &&
                  (S.scalar_type() == at::kBFloat16 || S.scalar_type() == at::kFloat),
              "soft_ce: student logits must be a contiguous bf16 / fp32 (R, K) CUDA matrix");
  TORCH_CHECK(T.is_cuda() && T.scalar_type() == at::kFloat && T.dim() == 2 && T.is_contiguous() &&
                  T.size(1) == S.size(1),
              "soft_ce: teacher probabilities must be a contiguous fp32 (Rt, K) matrix");
  TORCH_CHECK(S.size(1) % 8 == 0, "soft_ce: K must be a multiple of 8");
  TORCH_CHECK(tidx.scalar_type() == at::kInt && tidx.is_contiguous() && tidx.dim() == 2 && tidx.size(0) == S.size(0) &&
                  tidx.size(1) >= 1 && tidx.size(1) <= kMaxPairs,
              "soft_ce: pair table must be int32 (R, n) with 1 <= n <= ", kMaxPairs);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.sizes() == tidx.sizes(),
              "soft_ce: pair weights must be fp32 with the pair table's shape");
}

}  // namespace

// lse (R,), loss (R,) fp32 outputs.
void soft_ce_fwd(at::Tensor S, at::Tensor T, at::Tensor tidx, at::Tensor w, double tau, at::Tensor lse, at::Tensor loss) {
  check_ce(S, T, tidx, w);
  c10::cuda::CUDAGuard guard(S.device());
  const int R = (int)S.size(0), K = (int)S.size(1), n = (int)tidx.size(1);
  if (R == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (S.scalar_type() == at::kBFloat16)
    soft_ce_fwd_kernel<__nv_bfloat16><<<R, kCeThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(S.data_ptr()), T.data_ptr<float>(), tidx.data_ptr<int>(),
        w.data_ptr<float>(), n, K, (float)(1.0 / tau), lse.data_ptr<float>(), loss.data_ptr<float>());
  else
    soft_ce_fwd_kernel<float><<<R, kCeThreads, 0, st>>>(S.data_ptr<float>(), T.data_ptr<float>(), tidx.data_ptr<int>(),
                                                        w.data_ptr<float>(), n, K, (float)(1.0 / tau),
                                                        lse.data_ptr<float>(), loss.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dS (R, K) in S's dtype; grad_scale: 1-element fp32 device tensor (upstream gradient of sum_i loss_i).
void soft_ce_bwd(at::Tensor S, at::Tensor T, at::Tensor tidx, at::Tensor w, double tau, at::Tensor lse,
                 at::Tensor grad_scale, at::Tensor dS) {
  check_ce(S, T, tidx, w);
  TORCH_CHECK(dS.scalar_type() == S.scalar_type() && dS.sizes() == S.sizes() && dS.is_contiguous(),
              "soft_ce_bwd: dS must match S");
  c10::cuda::CUDAGuard guard(S.device());
  const int R = (int)S.size(0), K = (int)S.size(1), n = (int)tidx.size(1);
  if (R == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (S.scalar_type() == at::kBFloat16)
    soft_ce_bwd_kernel<__nv_bfloat16><<<R, kCeThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(S.data_ptr()), T.data_ptr<float>(), tidx.data_ptr<int>(),
        w.data_ptr<float>(), n, K, (float)(1.0 / tau), lse.data_ptr<float>(), grad_scale.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dS.data_ptr()));
  else
    soft_ce_bwd_kernel<float><<<R, kCeThreads, 0, st>>>(S.data_ptr<float>(), T.data_ptr<float>(), tidx.data_ptr<int>(),
                                                        w.data_ptr<float>(), n, K, (float)(1.0 / tau),
                                                        lse.data_ptr<float>(), grad_scale.data_ptr<float>(),
                                                        dS.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x (B, D) fp32 contiguous; outputs xn (B, D), nn (B,) int32, dist (B,), loss (1,).
void koleo_fwd(at::Tensor x, double eps, at::Tensor xn, at::Tensor nn, at::Tensor dist, at::Tensor loss) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.dim() == 2 && x.is_contiguous(),
              "koleo: fp32 contiguous (B, D) CUDA rows expected");
  const int B = (int)x.size(0), D = (int)x.size(1);
  TORCH_CHECK(B >= 2 && B <= 8192, "koleo: 2..8192 rows");
  c10::cuda::CUDAGuard guard(x.device());
  koleo_fwd_kernel<<<1, kKoleoThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), B, D, (float)eps, xn.data_ptr<float>(), nn.data_ptr<int>(), dist.data_ptr<float>(),
      loss.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void koleo_bwd(at::Tensor x, at::Tensor xn, at::Tensor nn, at::Tensor dist, double eps, at::Tensor grad,
               at::Tensor dxn, at::Tensor dx) {
  const int B = (int)x.size(0), D = (int)x.size(1);
  c10::cuda::CUDAGuard guard(x.device());
  koleo_bwd_kernel<<<1, kKoleoThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), xn.data_ptr<float>(), nn.data_ptr<int>(), dist.data_ptr<float>(), B, D, (float)eps,
      grad.data_ptr<float>(), dxn.data_ptr<float>(), dx.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
