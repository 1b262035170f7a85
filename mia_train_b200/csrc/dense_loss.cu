// Fused dense-prediction losses for volumetric segmentation heads.
//
// affinity_bce: affinity targets are never materialised. For voxel p and channel c with offset o_c
// the target is (label[p] == label[p + o_c]) && label[p] > 0 and the loss mask is "p + o_c inside
// the crop and neither label equals ignore_index" (reference semantics:
// src/algorithms/affinity/targets.py:213-260 and src/algorithms/affinity_seg.py:298-323). One
// forward pass reads the logits and labels once and produces six sums (masked BCE, mask count,
// correct, positive, cut, cut-correct); the backward pass recomputes the target on the fly and
// writes (sigmoid(x) - t) * m * g / count.
//
// semantic_ce: per-voxel softmax cross-entropy over K classes with optional class weights and an
// ignore index (torch weighted-mean semantics), plus argmax and a per-class intersection /
// prediction / label histogram, in one pass (reference src/algorithms/semantic_seg.py:194-217).
// The backward writes (softmax - onehot) * w[y] * g / sum(w[y]).
//
// Both are thread-per-voxel over the fastest spatial axis (coalesced per channel plane), with
// block reductions in shared memory and one double atomic per statistic per block.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace mia {

namespace {

constexpr int kMaxAffinityChannels = 32;

struct AffinityOffsets {
  int n;
  int d[kMaxAffinityChannels][3];
};

template <typename T>
__device__ __forceinline__ float to_f(T v) { return static_cast<float>(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v) { return static_cast<T>(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

__device__ __forceinline__ float bce_logits(float x, float t) {
  // max(x, 0) - x t + log(1 + exp(-|x|)), the overflow-free form
  return fmaxf(x, 0.f) - x * t + log1pf(expf(-fabsf(x)));
}

template <int N>
__device__ __forceinline__ void block_reduce_add(float (&v)[N], double* out) {
  __shared__ float red[N][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[i][warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float s = lane < nw ? red[i][lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0 && s != 0.f) atomicAdd(out + i, (double)s);
    }
  }
}

template <typename T, typename L>
__global__ void affinity_bce_fwd_kernel(const T* __restrict__ logits, const L* __restrict__ labels, int64_t batch,
                                        int X, int Y, int Z, AffinityOffsets offs, int64_t ignore,
                                        double* __restrict__ sums) {
  const int64_t S = (int64_t)X * Y * Z;
  const int64_t total = batch * S;
  float acc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / S;
    const int64_t p = idx - b * S;
    const int z = (int)(p % Z);
    const int y = (int)((p / Z) % Y);
    const int x = (int)(p / ((int64_t)Y * Z));
    const L* lab = labels + b * S;
    const int64_t a = (int64_t)lab[p];
    const T* lg = logits + b * (int64_t)offs.n * S + p;
    for (int c = 0; c < offs.n; ++c) {
      const int qx = x + offs.d[c][0], qy = y + offs.d[c][1], qz = z + offs.d[c][2];
      if (qx < 0 || qx >= X || qy < 0 || qy >= Y || qz < 0 || qz >= Z) continue;
      const int64_t nb = (int64_t)lab[((int64_t)qx * Y + qy) * Z + qz];
      if (a == ignore || nb == ignore) continue;
      const float t = (a == nb && a > 0) ? 1.f : 0.f;
      const float v = to_f(lg[(int64_t)c * S]);
      acc[0] += bce_logits(v, t);
      acc[1] += 1.f;
      const bool correct = (v > 0.f) == (t > 0.5f);
      acc[2] += correct ? 1.f : 0.f;
      acc[3] += t;
      if (t < 0.5f) {
        acc[4] += 1.f;
        acc[5] += correct ? 1.f : 0.f;
      }
    }
  }
  block_reduce_add<6>(acc, sums);
}

template <typename T, typename L>
__global__ void affinity_bce_bwd_kernel(const T* __restrict__ logits, const L* __restrict__ labels, int64_t batch,
                                        int X, int Y, int Z, AffinityOffsets offs, int64_t ignore,
                                        const double* __restrict__ sums, const float* __restrict__ grad_out,
                                        T* __restrict__ grad) {
  const int64_t S = (int64_t)X * Y * Z;
  const int64_t total = batch * S;
  const float scale = grad_out[0] / (float)fmax(sums[1], 1.0);
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / S;
    const int64_t p = idx - b * S;
    const int z = (int)(p % Z);
    const int y = (int)((p / Z) % Y);
    const int x = (int)(p / ((int64_t)Y * Z));
    const L* lab = labels + b * S;
    const int64_t a = (int64_t)lab[p];
    const int64_t base = b * (int64_t)offs.n * S + p;
    for (int c = 0; c < offs.n; ++c) {
      const int qx = x + offs.d[c][0], qy = y + offs.d[c][1], qz = z + offs.d[c][2];
      float g = 0.f;
      if (!(qx < 0 || qx >= X || qy < 0 || qy >= Y || qz < 0 || qz >= Z)) {
        const int64_t nb = (int64_t)lab[((int64_t)qx * Y + qy) * Z + qz];
        if (a != ignore && nb != ignore) {
          const float t = (a == nb && a > 0) ? 1.f : 0.f;
          const float v = to_f(logits[base + (int64_t)c * S]);
          g = (1.f / (1.f + expf(-v)) - t) * scale;
        }
      }
      grad[base + (int64_t)c * S] = from_f<T>(g);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// semantic cross-entropy + confusion statistics
// stats: [0] sum w[y] * nll, [1] sum w[y], [2] valid voxels, [3] correct voxels
// hist (3, K) int64 as doubles: [0] intersection, [1] predicted count, [2] label count (valid only)
template <typename T>
__global__ void semantic_ce_fwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ labels, int64_t batch,
                                       int64_t S, int K, const float* __restrict__ weights, int64_t ignore,
                                       double* __restrict__ stats, double* __restrict__ hist) {
  extern __shared__ float sh_hist[];  // 3 * K
  for (int i = threadIdx.x; i < 3 * K; i += blockDim.x) sh_hist[i] = 0.f;
  __syncthreads();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t total = batch * S;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / S;
    const int64_t p = idx - b * S;
    const int64_t y = labels[idx];
    if (y == ignore) continue;
    if (y < 0 || y >= K) continue;  // out-of-vocabulary label: not counted (the host checks the range)
    const T* lg = logits + b * (int64_t)K * S + p;
    // one pass: running max, rescaled exp-sum and argmax (first maximum wins, as torch.argmax)
    float mx = to_f(lg[0]);
    float se = 1.f;
    int arg = 0;
    for (int k = 1; k < K; ++k) {
      const float v = to_f(lg[(int64_t)k * S]);
      if (v > mx) {
        se = se * expf(mx - v) + 1.f;
        mx = v;
        arg = k;
      } else {
        se += expf(v - mx);
      }
    }
    const float nll = logf(se) + mx - to_f(lg[y * S]);
    const float w = weights ? weights[y] : 1.f;
    acc[0] += w * nll;
    acc[1] += w;
    acc[2] += 1.f;
    acc[3] += (arg == (int)y) ? 1.f : 0.f;
    if (arg == (int)y) atomicAdd(&sh_hist[arg], 1.f);
    atomicAdd(&sh_hist[K + arg], 1.f);
    atomicAdd(&sh_hist[2 * K + (int)y], 1.f);
  }
  block_reduce_add<4>(acc, stats);
  __syncthreads();
  for (int i = threadIdx.x; i < 3 * K; i += blockDim.x)
    if (sh_hist[i] != 0.f) atomicAdd(hist + i, (double)sh_hist[i]);
}

template <typename T>
__global__ void semantic_ce_bwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ labels, int64_t batch,
                                       int64_t S, int K, const float* __restrict__ weights, int64_t ignore,
                                       const double* __restrict__ stats, const float* __restrict__ grad_out,
                                       T* __restrict__ grad) {
  const int64_t total = batch * S;
  const float scale = grad_out[0] / (float)stats[1];
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / S;
    const int64_t p = idx - b * S;
    const int64_t y = labels[idx];
    const int64_t base = b * (int64_t)K * S + p;
    if (y == ignore || y < 0 || y >= K) {
      for (int k = 0; k < K; ++k) grad[base + (int64_t)k * S] = from_f<T>(0.f);
      continue;
    }
    float mx = -INFINITY;
    for (int k = 0; k < K; ++k) mx = fmaxf(mx, to_f(logits[base + (int64_t)k * S]));
    float se = 0.f;
    for (int k = 0; k < K; ++k) se += expf(to_f(logits[base + (int64_t)k * S]) - mx);
    const float inv = 1.f / se;
    const float w = (weights ? weights[y] : 1.f) * scale;
    for (int k = 0; k < K; ++k) {
      const float pk = expf(to_f(logits[base + (int64_t)k * S]) - mx) * inv;
      grad[base + (int64_t)k * S] = from_f<T>((pk - (k == (int)y ? 1.f : 0.f)) * w);
    }
  }
}

int grid_for(int64_t total, int threads) {
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const int64_t need = (total + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)sms * 8));
}

AffinityOffsets make_offsets(const std::vector<int64_t>& flat) {
  TORCH_CHECK(flat.size() % 3 == 0, "affinity offsets: expected a flat list of (dx, dy, dz) triples");
  AffinityOffsets o{};
  o.n = (int)(flat.size() / 3);
  TORCH_CHECK(o.n >= 1 && o.n <= kMaxAffinityChannels, "affinity offsets: 1..", kMaxAffinityChannels, " channels");
  for (int c = 0; c < o.n; ++c)
    for (int j = 0; j < 3; ++j) o.d[c][j] = (int)flat[3 * c + j];
  return o;
}

void check_affinity_inputs(const at::Tensor& logits, const at::Tensor& labels, const AffinityOffsets& o) {
  TORCH_CHECK(logits.is_cuda() && labels.is_cuda(), "affinity_bce: CUDA tensors expected");
  TORCH_CHECK(logits.dim() == 5 && labels.dim() == 4, "affinity_bce: logits (B, C, X, Y, Z), labels (B, X, Y, Z)");
  TORCH_CHECK(logits.is_contiguous() && labels.is_contiguous(), "affinity_bce: contiguous tensors expected");
  TORCH_CHECK(logits.size(1) == o.n, "affinity_bce: logits carry ", logits.size(1), " channels but ", o.n, " offsets were given");
  TORCH_CHECK(logits.size(0) == labels.size(0) && logits.size(2) == labels.size(1) && logits.size(3) == labels.size(2) &&
                  logits.size(4) == labels.size(3),
              "affinity_bce: logits and labels must share batch and spatial shape");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "affinity_bce: bf16 or fp32 logits");
  TORCH_CHECK(labels.scalar_type() == at::kLong || labels.scalar_type() == at::kInt, "affinity_bce: int64 or int32 labels");
}

}  // namespace

at::Tensor affinity_bce_fwd(at::Tensor logits, at::Tensor labels, std::vector<int64_t> offsets, int64_t ignore_index) {
  const AffinityOffsets o = make_offsets(offsets);
  check_affinity_inputs(logits, labels, o);
  c10::cuda::CUDAGuard guard(logits.device());
  auto sums = at::zeros({6}, logits.options().dtype(at::kDouble));
  const int X = (int)labels.size(1), Y = (int)labels.size(2), Z = (int)labels.size(3);
  const int64_t total = labels.numel();
  if (total == 0) return sums;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const int grid = grid_for(total, threads);
#define MIA_AFF_FWD(T, L)                                                                                      \
  affinity_bce_fwd_kernel<T, L><<<grid, threads, 0, stream>>>(                                                 \
      reinterpret_cast<const T*>(logits.data_ptr()), labels.data_ptr<L>(), labels.size(0), X, Y, Z, o,         \
      ignore_index, sums.data_ptr<double>())
  if (logits.scalar_type() == at::kBFloat16) {
    if (labels.scalar_type() == at::kLong) MIA_AFF_FWD(__nv_bfloat16, int64_t); else MIA_AFF_FWD(__nv_bfloat16, int32_t);
  } else {
    if (labels.scalar_type() == at::kLong) MIA_AFF_FWD(float, int64_t); else MIA_AFF_FWD(float, int32_t);
  }
#undef MIA_AFF_FWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return sums;
}

at::Tensor affinity_bce_bwd(at::Tensor logits, at::Tensor labels, std::vector<int64_t> offsets, int64_t ignore_index,
                            at::Tensor sums, at::Tensor grad_out) {
  const AffinityOffsets o = make_offsets(offsets);
  check_affinity_inputs(logits, labels, o);
  TORCH_CHECK(sums.scalar_type() == at::kDouble && sums.numel() == 6, "affinity_bce_bwd: sums from the forward expected");
  TORCH_CHECK(grad_out.scalar_type() == at::kFloat && grad_out.numel() == 1 && grad_out.is_cuda(),
              "affinity_bce_bwd: fp32 scalar grad expected");
  c10::cuda::CUDAGuard guard(logits.device());
  auto grad = at::empty_like(logits);
  const int X = (int)labels.size(1), Y = (int)labels.size(2), Z = (int)labels.size(3);
  const int64_t total = labels.numel();
  if (total == 0) return grad;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const int grid = grid_for(total, threads);
#define MIA_AFF_BWD(T, L)                                                                                       \
  affinity_bce_bwd_kernel<T, L><<<grid, threads, 0, stream>>>(                                                  \
      reinterpret_cast<const T*>(logits.data_ptr()), labels.data_ptr<L>(), labels.size(0), X, Y, Z, o,          \
      ignore_index, sums.data_ptr<double>(), grad_out.data_ptr<float>(), reinterpret_cast<T*>(grad.data_ptr()))
  if (logits.scalar_type() == at::kBFloat16) {
    if (labels.scalar_type() == at::kLong) MIA_AFF_BWD(__nv_bfloat16, int64_t); else MIA_AFF_BWD(__nv_bfloat16, int32_t);
  } else {
    if (labels.scalar_type() == at::kLong) MIA_AFF_BWD(float, int64_t); else MIA_AFF_BWD(float, int32_t);
  }
#undef MIA_AFF_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return grad;
}

std::vector<at::Tensor> semantic_ce_fwd(at::Tensor logits, at::Tensor labels, c10::optional<at::Tensor> weights,
                                        int64_t ignore_index) {
  TORCH_CHECK(logits.is_cuda() && labels.is_cuda(), "semantic_ce: CUDA tensors expected");
  TORCH_CHECK(logits.is_contiguous() && labels.is_contiguous() && labels.scalar_type() == at::kLong,
              "semantic_ce: contiguous logits and int64 labels expected");
  TORCH_CHECK(logits.dim() == labels.dim() + 1, "semantic_ce: logits (B, K, *S), labels (B, *S)");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "semantic_ce: bf16 or fp32 logits");
  const int64_t B = logits.size(0);
  const int K = (int)logits.size(1);
  TORCH_CHECK(K >= 1 && K <= 4096, "semantic_ce: 1..4096 classes");
  const int64_t S = labels.numel() / std::max<int64_t>(B, 1);
  TORCH_CHECK(logits.numel() == B * K * S, "semantic_ce: logits and labels shapes disagree");
  const float* w = nullptr;
  if (weights.has_value() && weights->defined()) {
    TORCH_CHECK(weights->scalar_type() == at::kFloat && weights->numel() == K && weights->is_contiguous() && weights->is_cuda(),
                "semantic_ce: fp32 class weights of length K expected");
    w = weights->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(logits.device());
  auto stats = at::zeros({4}, logits.options().dtype(at::kDouble));
  auto hist = at::zeros({3, K}, logits.options().dtype(at::kDouble));
  const int64_t total = B * S;
  if (total == 0) return {stats, hist};
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const int grid = grid_for(total, threads);
  const size_t smem = 3 * (size_t)K * sizeof(float);
  if (logits.scalar_type() == at::kBFloat16)
    semantic_ce_fwd_kernel<__nv_bfloat16><<<grid, threads, smem, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), labels.data_ptr<int64_t>(), B, S, K, w, ignore_index,
        stats.data_ptr<double>(), hist.data_ptr<double>());
  else
    semantic_ce_fwd_kernel<float><<<grid, threads, smem, stream>>>(logits.data_ptr<float>(), labels.data_ptr<int64_t>(), B,
                                                                   S, K, w, ignore_index, stats.data_ptr<double>(),
                                                                   hist.data_ptr<double>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {stats, hist};
}

at::Tensor semantic_ce_bwd(at::Tensor logits, at::Tensor labels, c10::optional<at::Tensor> weights, int64_t ignore_index,
                           at::Tensor stats, at::Tensor grad_out) {
  const int64_t B = logits.size(0);
  const int K = (int)logits.size(1);
  const int64_t S = labels.numel() / std::max<int64_t>(B, 1);
  const float* w = nullptr;
  if (weights.has_value() && weights->defined()) w = weights->data_ptr<float>();
  TORCH_CHECK(grad_out.scalar_type() == at::kFloat && grad_out.numel() == 1, "semantic_ce_bwd: fp32 scalar grad expected");
  c10::cuda::CUDAGuard guard(logits.device());
  auto grad = at::empty_like(logits);
  const int64_t total = B * S;
  if (total == 0) return grad;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const int grid = grid_for(total, threads);
  if (logits.scalar_type() == at::kBFloat16)
    semantic_ce_bwd_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), labels.data_ptr<int64_t>(), B, S, K, w, ignore_index,
        stats.data_ptr<double>(), grad_out.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()));
  else
    semantic_ce_bwd_kernel<float><<<grid, threads, 0, stream>>>(logits.data_ptr<float>(), labels.data_ptr<int64_t>(), B, S,
                                                                K, w, ignore_index, stats.data_ptr<double>(),
                                                                grad_out.data_ptr<float>(), grad.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return grad;
}

}  // namespace mia
