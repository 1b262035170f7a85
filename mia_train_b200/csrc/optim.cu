// Multi-tensor optimizer kernels over a device table of tensor pointers.
//
// * multi_tensor_sumsq: out += sum of squares of every element of every tensor (fp32 or bf16).
// * multi_tensor_scale: every tensor *= coef[0] (a device scalar, so a clip needs no host sync).
// * adamw_step: torch.optim.AdamW's update for fp32 params/moments with fp32 grads, per-tensor
//   device step counters and per-group (lr, weight_decay, beta1, beta2); an optional device
//   `grad_scale` multiplies each gradient as it is read. A second tiny launch increments the steps
//   afterwards, so every CTA of a tensor sees the same step.
//
// The pointer tables are cached per tensor list (keyed by addresses and sizes), so a CUDA graph
// capturing these launches replays them without any host work.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace mia {

constexpr int kChunk = 32768;  // elements per CTA

struct TensorEntry {
  void* ptr[6];
  int64_t numel;
  int32_t group;
  int32_t dtype;  // 0 fp32, 1 bf16 (for the first pointer)
};

struct Table {
  at::Tensor entries;  // device, TensorEntry[]
  at::Tensor chunks;   // device, int2[] (tensor index, chunk index)
  at::Tensor host_entries;
  at::Tensor host_chunks;
  int num_chunks = 0;
  int num_tensors = 0;
};

static std::mutex g_table_lock;
// Heap-allocated and never destroyed: its tensors must not be freed after the CUDA context is gone
// at process exit.
static std::map<std::vector<int64_t>, Table>& g_tables = *new std::map<std::vector<int64_t>, Table>();

static const Table& get_table(const std::vector<std::vector<at::Tensor>>& lists, const at::Tensor* groups) {
  const auto& first = lists[0];
  std::vector<int64_t> key;
  key.reserve(first.size() * (lists.size() + 1) + 2);
  key.push_back((int64_t)lists.size());
  key.push_back(first.empty() ? -1 : first[0].get_device());
  for (auto& l : lists) key.push_back((int64_t)l.size());
  for (size_t i = 0; i < first.size(); ++i) {
    key.push_back(first[i].numel());
    for (auto& l : lists) key.push_back((int64_t)reinterpret_cast<uintptr_t>(l[i].data_ptr()));
  }
  if (groups) key.push_back((int64_t)reinterpret_cast<uintptr_t>(groups->data_ptr()));
  std::lock_guard<std::mutex> guard(g_table_lock);
  auto it = g_tables.find(key);
  if (it != g_tables.end()) return it->second;
  if (g_tables.size() > 256) g_tables.clear();  // tensors were reallocated; drop stale tables
  Table t;
  t.num_tensors = (int)first.size();
  t.host_entries = at::empty({(int64_t)(first.size() * sizeof(TensorEntry))}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
  auto* e = reinterpret_cast<TensorEntry*>(t.host_entries.data_ptr());
  std::vector<int32_t> chunk_list;
  at::Tensor groups_cpu = groups ? groups->to(at::kCPU) : at::Tensor();
  for (size_t i = 0; i < first.size(); ++i) {
    for (int j = 0; j < 6; ++j)
      e[i].ptr[j] = (j < (int)lists.size() && lists[j][i].numel() > 0) ? lists[j][i].data_ptr() : nullptr;
    e[i].numel = first[i].numel();
    e[i].group = groups ? groups_cpu.data_ptr<int32_t>()[i] : 0;
    e[i].dtype = first[i].scalar_type() == at::kBFloat16 ? 1 : 0;
    const int64_t nch = (e[i].numel + kChunk - 1) / kChunk;
    for (int64_t c = 0; c < nch; ++c) {
      chunk_list.push_back((int32_t)i);
      chunk_list.push_back((int32_t)c);
    }
  }
  t.num_chunks = (int)(chunk_list.size() / 2);
  t.host_chunks = at::empty({(int64_t)chunk_list.size()}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
  std::memcpy(t.host_chunks.data_ptr(), chunk_list.data(), chunk_list.size() * 4);
  auto dev = first[0].device();
  t.entries = t.host_entries.to(dev, /*non_blocking=*/true);
  t.chunks = t.host_chunks.to(dev, /*non_blocking=*/true);
  return g_tables.emplace(key, std::move(t)).first->second;
}

__global__ void sumsq_kernel(const TensorEntry* __restrict__ entries, const int2* __restrict__ chunks,
                             float* __restrict__ out) {
  const int2 ch = chunks[blockIdx.x];
  const TensorEntry e = entries[ch.x];
  const int64_t start = (int64_t)ch.y * kChunk;
  const int64_t end = min(e.numel, start + kChunk);
  float s = 0.f;
  if (e.dtype == 0) {
    const float* p = reinterpret_cast<const float*>(e.ptr[0]);
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
      const float v = p[i];
      s += v * v;
    }
  } else {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(e.ptr[0]);
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
      const float v = __bfloat162float(p[i]);
      s += v * v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float warp_sums[32];
  if (threadIdx.x % 32 == 0) warp_sums[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) tot += warp_sums[w];
    atomicAdd(out, tot);
  }
}

__global__ void scale_kernel(const TensorEntry* __restrict__ entries, const int2* __restrict__ chunks,
                             const float* __restrict__ coef) {
  const int2 ch = chunks[blockIdx.x];
  const TensorEntry e = entries[ch.x];
  const int64_t start = (int64_t)ch.y * kChunk;
  const int64_t end = min(e.numel, start + kChunk);
  const float c = *coef;
  if (e.dtype == 0) {
    float* p = reinterpret_cast<float*>(e.ptr[0]);
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) p[i] *= c;
  } else {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(e.ptr[0]);
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) p[i] = __float2bfloat16_rn(__bfloat162float(p[i]) * c);
  }
}

// entries: ptr = {param, grad, exp_avg, exp_avg_sq, step, bf16 shadow (optional)}
__global__ void adamw_kernel(const TensorEntry* __restrict__ entries, const int2* __restrict__ chunks,
                             const float4* __restrict__ hyper, float eps, const float* __restrict__ grad_scale) {
  const int2 ch = chunks[blockIdx.x];
  const TensorEntry e = entries[ch.x];
  const float4 hp = hyper[e.group];  // lr, wd, beta1, beta2
  const float lr = hp.x, wd = hp.y, b1 = hp.z, b2 = hp.w;
  const float step = *reinterpret_cast<const float*>(e.ptr[4]) + 1.0f;
  const float bc1 = 1.0f - powf(b1, step);
  const float bc2_sqrt = sqrtf(1.0f - powf(b2, step));
  const float step_size = lr / bc1;
  const float decay = 1.0f - lr * wd;
  const float gs = grad_scale != nullptr ? *grad_scale : 1.0f;
  float* p = reinterpret_cast<float*>(e.ptr[0]);
  const float* gr = reinterpret_cast<const float*>(e.ptr[1]);
  float* m = reinterpret_cast<float*>(e.ptr[2]);
  float* v = reinterpret_cast<float*>(e.ptr[3]);
  __nv_bfloat16* shadow = reinterpret_cast<__nv_bfloat16*>(e.ptr[5]);
  const int64_t start = (int64_t)ch.y * kChunk;
  const int64_t end = min(e.numel, start + kChunk);
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(gr) | reinterpret_cast<uintptr_t>(m) |
                     reinterpret_cast<uintptr_t>(v)) & 15) == 0 &&
                   (shadow == nullptr || (reinterpret_cast<uintptr_t>(shadow) & 7) == 0);
  int64_t vec_end = start;
  if (vec) {
    vec_end = start + ((end - start) / 4) * 4;
    for (int64_t i = start + 4 * threadIdx.x; i < vec_end; i += 4 * blockDim.x) {
      float4 g4 = *reinterpret_cast<const float4*>(gr + i);
      float4 p4 = *reinterpret_cast<const float4*>(p + i);
      float4 m4 = *reinterpret_cast<const float4*>(m + i);
      float4 v4 = *reinterpret_cast<const float4*>(v + i);
      float gg[4] = {g4.x, g4.y, g4.z, g4.w}, pp[4] = {p4.x, p4.y, p4.z, p4.w};
      float mm[4] = {m4.x, m4.y, m4.z, m4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g = gg[j] * gs;
        mm[j] = mm[j] + (1.0f - b1) * (g - mm[j]);
        vv[j] = vv[j] * b2 + (1.0f - b2) * g * g;
        pp[j] = pp[j] * decay - step_size * (mm[j] / (sqrtf(vv[j]) / bc2_sqrt + eps));
      }
      *reinterpret_cast<float4*>(p + i) = make_float4(pp[0], pp[1], pp[2], pp[3]);
      *reinterpret_cast<float4*>(m + i) = make_float4(mm[0], mm[1], mm[2], mm[3]);
      *reinterpret_cast<float4*>(v + i) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      if (shadow != nullptr)
        *reinterpret_cast<uint2*>(shadow + i) = make_uint2(pack_bf16x2(pp[0], pp[1]), pack_bf16x2(pp[2], pp[3]));
    }
  }
  for (int64_t i = vec_end + threadIdx.x; i < end; i += blockDim.x) {
    const float g = gr[i] * gs;
    float pi = p[i] * decay;
    float mi = m[i];
    mi = mi + (1.0f - b1) * (g - mi);
    float vi = v[i] * b2 + (1.0f - b2) * g * g;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    pi = pi - step_size * (mi / denom);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (shadow != nullptr) shadow[i] = __float2bfloat16_rn(pi);
  }
}

// teacher = momentum * teacher + (1 - momentum) * student; entries: ptr = {teacher, student}.
__global__ void ema_kernel(const TensorEntry* __restrict__ entries, const int2* __restrict__ chunks, float momentum) {
  const int2 ch = chunks[blockIdx.x];
  const TensorEntry e = entries[ch.x];
  float* t = reinterpret_cast<float*>(e.ptr[0]);
  const float* s = reinterpret_cast<const float*>(e.ptr[1]);
  const int64_t start = (int64_t)ch.y * kChunk;
  const int64_t end = min(e.numel, start + kChunk);
  const float a = 1.0f - momentum;
  if (((reinterpret_cast<uintptr_t>(t) | reinterpret_cast<uintptr_t>(s)) & 15) == 0) {
    const int64_t vend = start + ((end - start) / 4) * 4;
    for (int64_t i = start + 4 * threadIdx.x; i < vend; i += 4 * blockDim.x) {
      float4 tv = *reinterpret_cast<float4*>(t + i);
      const float4 sv = *reinterpret_cast<const float4*>(s + i);
      tv.x = momentum * tv.x + a * sv.x;
      tv.y = momentum * tv.y + a * sv.y;
      tv.z = momentum * tv.z + a * sv.z;
      tv.w = momentum * tv.w + a * sv.w;
      *reinterpret_cast<float4*>(t + i) = tv;
    }
    for (int64_t i = vend + threadIdx.x; i < end; i += blockDim.x) t[i] = momentum * t[i] + a * s[i];
  } else {
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) t[i] = momentum * t[i] + a * s[i];
  }
}

__global__ void increment_steps_kernel(const TensorEntry* __restrict__ entries, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) *reinterpret_cast<float*>(entries[i].ptr[4]) += 1.0f;
}

void multi_tensor_sumsq(std::vector<at::Tensor> tensors, at::Tensor out) {
  if (tensors.empty()) return;
  c10::cuda::CUDAGuard guard(tensors[0].device());
  for (auto& t : tensors)
    TORCH_CHECK(t.is_cuda() && t.is_contiguous() && (t.scalar_type() == at::kFloat || t.scalar_type() == at::kBFloat16),
                "multi_tensor_sumsq: contiguous fp32/bf16 CUDA tensors");
  const Table& tab = get_table({tensors}, nullptr);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  sumsq_kernel<<<tab.num_chunks, 256, 0, stream>>>(reinterpret_cast<const TensorEntry*>(tab.entries.data_ptr()),
                                                   reinterpret_cast<const int2*>(tab.chunks.data_ptr()),
                                                   out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ema_update(std::vector<at::Tensor> teacher, std::vector<at::Tensor> student, double momentum) {
  if (teacher.empty()) return;
  TORCH_CHECK(teacher.size() == student.size(), "ema_update: list lengths differ");
  for (size_t i = 0; i < teacher.size(); ++i)
    TORCH_CHECK(teacher[i].scalar_type() == at::kFloat && student[i].scalar_type() == at::kFloat &&
                    teacher[i].numel() == student[i].numel() && teacher[i].is_contiguous() && student[i].is_contiguous(),
                "ema_update: matching contiguous fp32 tensors expected");
  c10::cuda::CUDAGuard guard(teacher[0].device());
  const Table& tab = get_table({teacher, student}, nullptr);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  ema_kernel<<<tab.num_chunks, 256, 0, stream>>>(reinterpret_cast<const TensorEntry*>(tab.entries.data_ptr()),
                                                 reinterpret_cast<const int2*>(tab.chunks.data_ptr()), (float)momentum);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void multi_tensor_scale(std::vector<at::Tensor> tensors, at::Tensor coef) {
  if (tensors.empty()) return;
  c10::cuda::CUDAGuard guard(tensors[0].device());
  const Table& tab = get_table({tensors}, nullptr);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  scale_kernel<<<tab.num_chunks, 256, 0, stream>>>(reinterpret_cast<const TensorEntry*>(tab.entries.data_ptr()),
                                                   reinterpret_cast<const int2*>(tab.chunks.data_ptr()),
                                                   coef.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step(std::vector<at::Tensor> params, std::vector<at::Tensor> grads, std::vector<at::Tensor> exp_avgs,
                std::vector<at::Tensor> exp_avg_sqs, std::vector<at::Tensor> steps, at::Tensor group_index,
                at::Tensor hyper, double eps, c10::optional<at::Tensor> grad_scale, std::vector<at::Tensor> shadows) {
  if (params.empty()) return;
  const size_t n = params.size();
  TORCH_CHECK(grads.size() == n && exp_avgs.size() == n && exp_avg_sqs.size() == n && steps.size() == n,
              "adamw_step: list lengths differ");
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(params[i].scalar_type() == at::kFloat && grads[i].scalar_type() == at::kFloat &&
                    exp_avgs[i].scalar_type() == at::kFloat && exp_avg_sqs[i].scalar_type() == at::kFloat,
                "adamw_step: fp32 params, grads and moments expected");
    TORCH_CHECK(params[i].is_contiguous() && grads[i].is_contiguous() && exp_avgs[i].is_contiguous() &&
                    exp_avg_sqs[i].is_contiguous(),
                "adamw_step: contiguous tensors expected");
    TORCH_CHECK(steps[i].is_cuda() && steps[i].scalar_type() == at::kFloat && steps[i].numel() == 1,
                "adamw_step: device fp32 scalar steps expected");
  }
  c10::cuda::CUDAGuard guard(params[0].device());
  std::vector<std::vector<at::Tensor>> lists = {params, grads, exp_avgs, exp_avg_sqs, steps};
  if (!shadows.empty()) {
    TORCH_CHECK(shadows.size() == n, "adamw_step: one shadow (or an empty tensor) per parameter");
    for (size_t i = 0; i < n; ++i)
      TORCH_CHECK(shadows[i].numel() == 0 || (shadows[i].scalar_type() == at::kBFloat16 &&
                                               shadows[i].numel() == params[i].numel() && shadows[i].is_contiguous()),
                  "adamw_step: shadows must be contiguous bf16 copies of the parameters");
    lists.push_back(shadows);
  }
  const Table& tab = get_table(lists, &group_index);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const float* gs = grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr;
  adamw_kernel<<<tab.num_chunks, 256, 0, stream>>>(reinterpret_cast<const TensorEntry*>(tab.entries.data_ptr()),
                                                   reinterpret_cast<const int2*>(tab.chunks.data_ptr()),
                                                   reinterpret_cast<const float4*>(hyper.data_ptr<float>()),
                                                   (float)eps, gs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  increment_steps_kernel<<<(tab.num_tensors + 255) / 256, 256, 0, stream>>>(
      reinterpret_cast<const TensorEntry*>(tab.entries.data_ptr()), tab.num_tensors);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
