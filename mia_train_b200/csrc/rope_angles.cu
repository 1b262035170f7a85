// Axial RoPE angle table and its frequency gradient.
//
//   angles[r, p] = coords[r, axis(p)] * freq(p)                    r = token (B * N rows)
//   dfreq(p)    += sum_r dangles[r, p] * coords[r, axis(p)]
//
// The frequencies are one learnable vector per spatial axis (reference
// src/layers/common/rope.py:78-120); pair p belongs to axis a for chunk_start[a] <= p <
// chunk_start[a + 1]. The backward adds straight into each axis' gradient buffer (the parameter's
// main_grad when it has one), one atomic per pair per CTA after a shared-memory reduction over the
// CTA's rows.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace mia {

namespace {

constexpr int kMaxAxes = 4;
constexpr int kMaxPairs = 128;

struct AxisTable {
  int axes;
  int start[kMaxAxes + 1];
  const float* freq[kMaxAxes];
  float* dfreq[kMaxAxes];
};

__device__ __forceinline__ int axis_of(const AxisTable& t, int p) {
  int a = 0;
#pragma unroll
  for (int i = 1; i < kMaxAxes; ++i)
    if (i < t.axes && p >= t.start[i]) a = i;
  return a;
}

__device__ __forceinline__ const float* freq_ptr(const AxisTable& t, int a) {
  const float* r = t.freq[0];
#pragma unroll
  for (int i = 1; i < kMaxAxes; ++i) r = (a == i) ? t.freq[i] : r;
  return r;
}

__device__ __forceinline__ float* dfreq_ptr(const AxisTable& t, int a) {
  float* r = t.dfreq[0];
#pragma unroll
  for (int i = 1; i < kMaxAxes; ++i) r = (a == i) ? t.dfreq[i] : r;
  return r;
}

__device__ __forceinline__ int start_of(const AxisTable& t, int a) {
  int r = t.start[0];
#pragma unroll
  for (int i = 1; i < kMaxAxes; ++i) r = (a == i) ? t.start[i] : r;
  return r;
}

__global__ void axial_angles_fwd_kernel(const float* __restrict__ coords, const AxisTable t, int64_t rows, int P,
                                        int A, float* __restrict__ angles) {
  const int64_t total = rows * P;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / P;
    const int p = (int)(i - r * P);
    const int a = axis_of(t, p);
    angles[i] = coords[r * A + a] * freq_ptr(t, a)[p - start_of(t, a)];
  }
}

// Block = 256 threads = 8 row-groups x 32 pair lanes (pairs p = lane, lane + 32, ...).
__global__ void axial_angles_bwd_kernel(const float* __restrict__ dangles, const float* __restrict__ coords,
                                        const AxisTable t, int64_t rows, int P, int A, int rows_per_cta) {
  __shared__ float part[8][kMaxPairs];
  const int lane = threadIdx.x % 32, group = threadIdx.x / 32;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);
  for (int p = lane; p < P; p += 32) {
    const int a = axis_of(t, p);
    float acc = 0.f;
    for (int64_t r = r0 + group; r < r1; r += 8) acc += dangles[r * P + p] * coords[r * A + a];
    part[group][p] = acc;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) s += part[g][p];
    const int a = axis_of(t, p);
    if (s != 0.f) atomicAdd(dfreq_ptr(t, a) + (p - start_of(t, a)), s);
  }
}

AxisTable make_table(const std::vector<at::Tensor>& freqs, const std::vector<at::Tensor>& dfreqs, int* P_out) {
  TORCH_CHECK(!freqs.empty() && (int)freqs.size() <= kMaxAxes, "axial_angles: 1..", kMaxAxes, " axes");
  AxisTable t{};
  t.axes = (int)freqs.size();
  int p = 0;
  for (int a = 0; a < t.axes; ++a) {
    TORCH_CHECK(freqs[a].scalar_type() == at::kFloat && freqs[a].is_contiguous() && freqs[a].dim() == 1,
                "axial_angles: contiguous fp32 frequency vectors");
    t.start[a] = p;
    t.freq[a] = freqs[a].data_ptr<float>();
    if (!dfreqs.empty()) {
      TORCH_CHECK(dfreqs[a].scalar_type() == at::kFloat && dfreqs[a].is_contiguous() &&
                      dfreqs[a].numel() == freqs[a].numel(),
                  "axial_angles: fp32 gradient buffers shaped like the frequencies");
      t.dfreq[a] = dfreqs[a].data_ptr<float>();
    }
    p += (int)freqs[a].numel();
  }
  for (int a = t.axes; a <= kMaxAxes; ++a) t.start[a] = p;
  TORCH_CHECK(p >= 1 && p <= kMaxPairs, "axial_angles: 1..", kMaxPairs, " pairs");
  *P_out = p;
  return t;
}

}  // namespace

at::Tensor axial_angles_fwd(at::Tensor coords, std::vector<at::Tensor> freqs) {
  TORCH_CHECK(coords.is_cuda() && coords.scalar_type() == at::kFloat && coords.is_contiguous(),
              "axial_angles: contiguous fp32 coordinates (..., A)");
  const int A = (int)coords.size(-1);
  TORCH_CHECK(A == (int)freqs.size(), "axial_angles: one frequency vector per coordinate axis");
  int P = 0;
  const AxisTable t = make_table(freqs, {}, &P);
  c10::cuda::CUDAGuard guard(coords.device());
  std::vector<int64_t> shape(coords.sizes().begin(), coords.sizes().end());
  shape.back() = P;
  auto angles = at::empty(shape, coords.options());
  const int64_t rows = coords.numel() / A;
  if (rows == 0) return angles;
  const int64_t total = rows * P;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 4096);
  axial_angles_fwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(coords.data_ptr<float>(), t, rows, P, A,
                                                                               angles.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return angles;
}

// dfreqs[a] += sum over rows (accumulates into the given buffers).
void axial_angles_bwd(at::Tensor dangles, at::Tensor coords, std::vector<at::Tensor> freqs,
                      std::vector<at::Tensor> dfreqs) {
  TORCH_CHECK(dangles.is_cuda() && dangles.scalar_type() == at::kFloat && dangles.is_contiguous(),
              "axial_angles_bwd: contiguous fp32 angle gradient");
  const int A = (int)coords.size(-1);
  TORCH_CHECK(dfreqs.size() == freqs.size(), "axial_angles_bwd: one gradient buffer per axis");
  int P = 0;
  const AxisTable t = make_table(freqs, dfreqs, &P);
  TORCH_CHECK(dangles.size(-1) == P, "axial_angles_bwd: angle gradient width must equal the pair count");
  c10::cuda::CUDAGuard guard(coords.device());
  const int64_t rows = coords.numel() / A;
  if (rows == 0) return;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const int rows_per_cta = (int)std::max<int64_t>(64, (rows + sms - 1) / sms);
  const int grid = (int)((rows + rows_per_cta - 1) / rows_per_cta);
  axial_angles_bwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      dangles.data_ptr<float>(), coords.data_ptr<float>(), t, rows, P, A, rows_per_cta);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
