// Peer-memory collectives for the sharded data-parallel optimizer step, over NVLink / NVSwitch.
//
// Memory: every rank allocates its buffers with cudaMalloc and exports them with CUDA IPC
// (`ipc_export`); the 64-byte handles are exchanged over the process group and opened on every
// peer (`ipc_open`), giving each rank a device pointer to every peer's copy. Kernels then move
// data with plain P2P loads and stores (no TMA, no multicast).
//
// Signalling: a per-rank flag area (int32) in IPC memory. A barrier slot is (kind, block, rank);
// a writer publishes `epoch` into the slot of every peer with a system-scope release store after
// its data stores and a system fence, a reader spins with system-scope acquire loads. Every spin
// is bounded by a %globaltimer deadline: on expiry the kernel records an error code in the
// per-device error word and returns (no trap), so the context stays usable and the host can read
// the failure. `epoch` is a device counter advanced once per step by `zero_advance_epoch`, so the
// whole step can be captured in a CUDA graph and replayed.
//
// The flat buffers are cut into segments; rank r owns the r-th slice of every segment. Kernels of
// one step (same grids on every rank, same order):
//   zero_reduce_scatter  -- per segment, possibly while backward still runs on later segments:
//                           start barrier (every rank finished that segment's gradients), then
//                           rank r sums its slice from every peer into its local gradient buffer
//                           and accumulates per-CTA sums of squares.
//   zero_norm_exchange   -- one CTA: local sum of squares -> every peer, barrier, global norm,
//                           clip coefficient (times 1/world) into a device scalar for AdamW.
//   (AdamW on the local shard: the multi-tensor kernel in optim.cu.)
//   zero_all_gather      -- per segment: push the updated slice to every peer (fp32 master values for the
//                           fp32 region, bf16 shadow values for the bf16 region), system fence,
//                           end barrier; then refresh the local copies of the other ranks' shards
//                           (bf16 region: fp32 <- bf16 shadow; fp32 region: shadow <- bf16(fp32)).
//
// Ordering argument: the start barrier of zero_reduce_scatter proves every peer finished its
// backward, so the peer gradients are complete and no peer reads parameters of this step any
// more; the end barrier of zero_all_gather proves every peer finished reading this rank's
// gradients (its reduce-scatter precedes its all-gather) and finished writing into this rank's
// parameters, so the next step may zero gradients and read parameters.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"
#include "errors.h"

namespace mia {

namespace {

constexpr int kMaxWorld = 8;
constexpr int kMaxBlocks = 512;
constexpr int kKinds = 4;  // 0 reduce-scatter start, 1 norm exchange, 2 all-gather end, 3 spare
constexpr int kFlagInts = kKinds * kMaxBlocks * kMaxWorld;
constexpr int kValueFloats = kMaxWorld;
// Barrier values are epoch * kSeqPerStep + seq + 1: `seq` numbers the launches of one kind within a
// step (all ranks launch them in the same order), so values only grow and a slot left over from an
// earlier launch can never satisfy a later one.
constexpr int kSeqPerStep = 128;

struct PeerPtrs {
  int64_t p[kMaxWorld];
};

// p.p[i] without a dynamic index into the parameter array (which would copy it to local memory).
__device__ __forceinline__ int64_t pick(const PeerPtrs p, int i) {
  int64_t r = p.p[0];
#pragma unroll
  for (int j = 1; j < kMaxWorld; ++j) r = (i == j) ? p.p[j] : r;
  return r;
}

__device__ __forceinline__ void st_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int* flag_slot(int64_t base, int kind, int block, int rank) {
  return reinterpret_cast<int*>(base) + ((kind * kMaxBlocks + block) * kMaxWorld + rank);
}

// Threads 0..world-1 of the block each signal one peer, then each wait for one peer.
// Returns false (after recording `code`) if a peer did not arrive before the deadline.
__device__ __forceinline__ bool block_barrier(const PeerPtrs flags, int kind, int rank, int world, int epoch, uint64_t timeout_ns,
                              int* err, int code) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  const int t = threadIdx.x;
  if (t < world) {
    st_release_sys(flag_slot(pick(flags, t), kind, blockIdx.x, rank), epoch);
    const int* mine = flag_slot(pick(flags, rank), kind, blockIdx.x, t);
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    while (ld_acquire_sys(mine) < epoch) {
      if (globaltimer_ns() > deadline) {
        record_error(err, code);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  return failed == 0;
}

__global__ void zero_reduce_scatter_kernel(PeerPtrs grads, PeerPtrs flags, int64_t shard_off, int64_t shard_len,
                                           float* __restrict__ partial, const int* __restrict__ epoch_ptr, int rank,
                                           int world, int seq, uint64_t timeout_ns, int* err) {
  const int epoch = *epoch_ptr * kSeqPerStep + seq + 1;
  float s = 0.f;
  if (block_barrier(flags, 0, rank, world, epoch, timeout_ns, err, kErrZeroReduceScatterWait)) {
    float* out = reinterpret_cast<float*>(pick(grads, rank)) + shard_off;
    const int64_t n4 = shard_len / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q) {
        if (q >= world) break;
        // start with a rotated peer so ranks spread their reads over different sources
        int p = rank + q;
        if (p >= world) p -= world;
        const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(pick(grads, p)) + shard_off)[i];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      reinterpret_cast<float4*>(out)[i] = acc;
      s += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
    partial[blockIdx.x] = tot;
  }
}

// The same reduce-scatter with bf16 on the wire. CTA b owns groups [g0, g1) of 8 elements of every
// shard of the segment: it first rounds this rank's fp32 gradient of that part of every shard to
// bf16 (this rank's IPC bf16 buffer), passes the per-block barrier (block b of every peer has
// rounded the same part of every shard, in particular of this rank's), then sums its part of this
// rank's shard from every rank's bf16 copy in fp32 into the local fp32 gradient and accumulates the
// sum of squares. Half the NVLink bytes of the fp32 kernel; the sum itself stays fp32.
__global__ void zero_reduce_scatter_bf16_kernel(PeerPtrs grads, PeerPtrs grads16, PeerPtrs flags, int64_t seg_lo,
                                                int64_t shard_len, float* __restrict__ partial,
                                                const int* __restrict__ epoch_ptr, int rank, int world, int seq,
                                                uint64_t timeout_ns, int* err) {
  const int epoch = *epoch_ptr * kSeqPerStep + seq + 1;
  const int64_t groups = shard_len / 8;
  const int64_t per = (groups + gridDim.x - 1) / gridDim.x;
  const int64_t g0 = blockIdx.x * per, g1 = min(groups, g0 + per);
  const float* my32 = reinterpret_cast<const float*>(pick(grads, rank));
  __nv_bfloat16* my16 = reinterpret_cast<__nv_bfloat16*>(pick(grads16, rank));
  for (int sh = 0; sh < world; ++sh) {
    const int64_t base = seg_lo + (int64_t)sh * shard_len;
    for (int64_t g = g0 + threadIdx.x; g < g1; g += blockDim.x) {
      const float4 a = *reinterpret_cast<const float4*>(my32 + base + g * 8);
      const float4 b = *reinterpret_cast<const float4*>(my32 + base + g * 8 + 4);
      *reinterpret_cast<uint4*>(my16 + base + g * 8) =
          make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
    }
  }
  __threadfence_system();
  float s = 0.f;
  if (block_barrier(flags, 0, rank, world, epoch, timeout_ns, err, kErrZeroReduceScatterWait)) {
    const int64_t own = seg_lo + (int64_t)rank * shard_len;
    float* out = reinterpret_cast<float*>(pick(grads, rank)) + own;
    for (int64_t g = g0 + threadIdx.x; g < g1; g += blockDim.x) {
      uint4 v[kMaxWorld];
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q) {
        int src = rank + q;
        if (src >= world) src -= world;  // rotated start spreads the reads over the sources
        if (q < world) v[q] = __ldcg(reinterpret_cast<const uint4*>(
                                  reinterpret_cast<const __nv_bfloat16*>(pick(grads16, src)) + own) + g);
      }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q) {
        if (q < world) {
          const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            acc[2 * h] += bf16_lo(w[h]);
            acc[2 * h + 1] += bf16_hi(w[h]);
          }
        }
      }
      *reinterpret_cast<float4*>(out + g * 8) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(out + g * 8 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += acc[j] * acc[j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
    partial[blockIdx.x] = tot;
  }
}

// values: float[kMaxWorld] area of every rank (inside the flag allocation, after the flags).
__global__ void zero_norm_exchange_kernel(PeerPtrs flags, const float* __restrict__ partial, int nparts,
                                          const int* __restrict__ epoch_ptr, int rank, int world, float max_norm,
                                          float* __restrict__ grad_scale, float* __restrict__ grad_norm,
                                          uint64_t timeout_ns, int* err) {
  const int epoch = *epoch_ptr * kSeqPerStep + 1;
  __shared__ float local_total;
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < nparts; ++i) t += partial[i];
    local_total = t;
  }
  __syncthreads();
  const int t = threadIdx.x;
  __shared__ int failed;
  if (t == 0) failed = 0;
  __syncthreads();
  if (t < world) {
    float* peer_values = reinterpret_cast<float*>(reinterpret_cast<int*>(pick(flags, t)) + kFlagInts);
    peer_values[rank] = local_total;
    __threadfence_system();
    st_release_sys(flag_slot(pick(flags, t), 1, 0, rank), epoch);
    const int* mine = flag_slot(pick(flags, rank), 1, 0, t);
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    while (ld_acquire_sys(mine) < epoch) {
      if (globaltimer_ns() > deadline) {
        record_error(err, kErrZeroNormWait);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (t == 0) {
    const float* values = reinterpret_cast<const float*>(reinterpret_cast<const int*>(pick(flags, rank)) + kFlagInts);
    float total = 0.f;
    for (int p = 0; p < world; ++p) total += values[p];
    // the averaged gradient is sum / world, so its norm is sqrt(sum of squares of sums) / world
    const float norm = sqrtf(total) / (float)world;
    float coef = 1.f;
    if (max_norm > 0.f) coef = fminf(1.f, max_norm / (norm + 1e-6f));
    if (failed) coef = 0.f;  // a missing peer: do not apply a partial gradient
    grad_norm[0] = norm;
    grad_scale[0] = coef / (float)world;
  }
}

// One segment [seg_lo, seg_lo + world * shard_len): rank r owns the r-th shard_len slice of it.
__global__ void zero_all_gather_kernel(PeerPtrs data, PeerPtrs shadow, PeerPtrs flags, int64_t seg_lo,
                                       int64_t shard_len, int64_t bf16_begin, const int* __restrict__ epoch_ptr,
                                       int rank, int world, int seq, uint64_t timeout_ns, int* err) {
  const int epoch = *epoch_ptr * kSeqPerStep + seq + 1;
  const int64_t own0 = seg_lo + (int64_t)rank * shard_len;
  // 1) push: groups of 8 elements (one uint4 of bf16, two float4 of fp32); bf16_begin and the
  //    shard bounds are multiples of 64, so a group never straddles the region boundary.
  const int64_t groups = shard_len / 8;
  const float* my_data = reinterpret_cast<const float*>(pick(data, rank));
  const __nv_bfloat16* my_shadow = reinterpret_cast<const __nv_bfloat16*>(pick(shadow, rank));
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = own0 + g * 8;
    if (e >= bf16_begin) {
      const uint4 v = *reinterpret_cast<const uint4*>(my_shadow + e);
      for (int q = 1; q < world; ++q) {
        int p = rank + q;
        if (p >= world) p -= world;
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(pick(shadow, p)) + e) = v;
      }
    } else {
      const float4 a = *reinterpret_cast<const float4*>(my_data + e);
      const float4 b = *reinterpret_cast<const float4*>(my_data + e + 4);
      for (int q = 1; q < world; ++q) {
        int p = rank + q;
        if (p >= world) p -= world;
        float* dst = reinterpret_cast<float*>(pick(data, p)) + e;
        *reinterpret_cast<float4*>(dst) = a;
        *reinterpret_cast<float4*>(dst + 4) = b;
      }
    }
  }
  __threadfence_system();
  if (!block_barrier(flags, 2, rank, world, epoch, timeout_ns, err, kErrZeroAllGatherWait)) return;
  // 2) refresh the local copies of the other shards; every block must finish its barrier first,
  //    so this phase only touches ranges whose writers this block has heard from: block b covers
  //    exactly the groups that block b of every peer wrote.
  float* d = reinterpret_cast<float*>(pick(data, rank));
  __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(pick(shadow, rank));
  for (int q = 1; q < world; ++q) {
    int p = rank + q;
    if (p >= world) p -= world;
    const int64_t base = seg_lo + (int64_t)p * shard_len;
    for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = base + g * 8;
      if (e >= bf16_begin) {
        const uint4 v = *reinterpret_cast<const uint4*>(sh + e);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
        float4 a, b;
        a.x = __bfloat162float(h[0]); a.y = __bfloat162float(h[1]); a.z = __bfloat162float(h[2]); a.w = __bfloat162float(h[3]);
        b.x = __bfloat162float(h[4]); b.y = __bfloat162float(h[5]); b.z = __bfloat162float(h[6]); b.w = __bfloat162float(h[7]);
        *reinterpret_cast<float4*>(d + e) = a;
        *reinterpret_cast<float4*>(d + e + 4) = b;
      } else {
        const float4 a = *reinterpret_cast<const float4*>(d + e);
        const float4 b = *reinterpret_cast<const float4*>(d + e + 4);
        uint4 v;
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&v);
        h[0] = __float2bfloat16(a.x); h[1] = __float2bfloat16(a.y); h[2] = __float2bfloat16(a.z); h[3] = __float2bfloat16(a.w);
        h[4] = __float2bfloat16(b.x); h[5] = __float2bfloat16(b.y); h[6] = __float2bfloat16(b.z); h[7] = __float2bfloat16(b.w);
        *reinterpret_cast<uint4*>(sh + e) = v;
      }
    }
  }
}

__global__ void zero_advance_epoch_kernel(int* epoch) { epoch[0] += 1; }

PeerPtrs to_peers(const std::vector<int64_t>& v, int world) {
  TORCH_CHECK((int)v.size() == world && world >= 1 && world <= kMaxWorld, "peer pointer list must have world (1..",
              kMaxWorld, ") entries");
  PeerPtrs p{};
  for (int i = 0; i < world; ++i) {
    TORCH_CHECK(v[i] != 0 && (v[i] & 15) == 0, "peer pointers must be non-null and 16-byte aligned");
    p.p[i] = v[i];
  }
  return p;
}

uint64_t timeout_from_ms(double ms) { return (uint64_t)(ms > 0 ? ms * 1e6 : 5e9); }

}  // namespace

// -------------------------------------------------------------------------------------------- IPC
std::vector<at::Tensor> ipc_export(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "ipc_export: positive size expected");
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, (size_t)nbytes));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, (size_t)nbytes));
  cudaIpcMemHandle_t handle;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&handle, ptr));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  // The tensor does not own the allocation: `ipc_free` releases it after every peer closed it.
  auto local = at::from_blob(ptr, {nbytes}, [](void*) {}, opts);
  auto h = at::empty({(int64_t)sizeof(handle)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(h.data_ptr(), &handle, sizeof(handle));
  auto addr = at::empty({1}, at::TensorOptions().dtype(at::kLong));
  addr.data_ptr<int64_t>()[0] = (int64_t)reinterpret_cast<uintptr_t>(ptr);
  return {local, h, addr};
}

std::vector<int64_t> ipc_open(at::Tensor handles, int64_t rank, int64_t local_ptr, int64_t device) {
  TORCH_CHECK(handles.device().is_cpu() && handles.scalar_type() == at::kByte && handles.dim() == 2 &&
                  handles.size(1) == (int64_t)sizeof(cudaIpcMemHandle_t),
              "ipc_open: (world, 64) uint8 CPU handles expected");
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  const int64_t world = handles.size(0);
  std::vector<int64_t> out(world, 0);
  for (int64_t r = 0; r < world; ++r) {
    if (r == rank) {
      out[r] = local_ptr;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].contiguous().data_ptr(), sizeof(h));
    void* ptr = nullptr;
    C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    out[r] = (int64_t)reinterpret_cast<uintptr_t>(ptr);
  }
  return out;
}

void ipc_close(std::vector<int64_t> peers, int64_t rank, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  for (int64_t r = 0; r < (int64_t)peers.size(); ++r)
    if (r != rank && peers[r] != 0) C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(peers[r])));
}

void ipc_free(int64_t local_ptr, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(local_ptr)));
}

int64_t comm_flag_bytes() { return (int64_t)(kFlagInts + kValueFloats) * 4; }

int64_t comm_max_blocks() { return kMaxBlocks; }

// ---------------------------------------------------------------------------------------- launches
void zero_reduce_scatter(std::vector<int64_t> grad_peers, std::vector<int64_t> flag_peers, int64_t shard_off,
                         int64_t shard_len, at::Tensor partial, at::Tensor epoch, int64_t rank, double timeout_ms,
                         int64_t seq, int64_t threads) {
  TORCH_CHECK(threads >= 64 && threads <= 1024 && threads % 32 == 0, "zero_reduce_scatter: 64..1024 threads, whole warps");
  TORCH_CHECK(seq >= 0 && seq < kSeqPerStep, "zero_reduce_scatter: launch sequence number out of range");
  const int world = (int)grad_peers.size();
  TORCH_CHECK(shard_off % 64 == 0 && shard_len % 64 == 0, "zero_reduce_scatter: shard must be 64-element aligned");
  TORCH_CHECK(partial.scalar_type() == at::kFloat && partial.is_cuda() && partial.numel() >= 1 &&
                  partial.numel() <= kMaxBlocks,
              "zero_reduce_scatter: partial sums buffer of 1..", kMaxBlocks, " floats expected");
  TORCH_CHECK(epoch.scalar_type() == at::kInt && epoch.is_cuda(), "zero_reduce_scatter: int32 device epoch expected");
  c10::cuda::CUDAGuard guard(partial.device());
  const int grid = (int)partial.numel();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  zero_reduce_scatter_kernel<<<grid, (int)threads, 0, stream>>>(to_peers(grad_peers, world), to_peers(flag_peers, world), shard_off,
                                                       shard_len, partial.data_ptr<float>(), epoch.data_ptr<int>(),
                                                       (int)rank, world, (int)seq, timeout_from_ms(timeout_ms),
                                                       error_word(partial.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void zero_reduce_scatter_bf16(std::vector<int64_t> grad_peers, std::vector<int64_t> grad16_peers,
                              std::vector<int64_t> flag_peers, int64_t seg_lo, int64_t shard_len, at::Tensor partial,
                              at::Tensor epoch, int64_t rank, double timeout_ms, int64_t seq, int64_t threads) {
  TORCH_CHECK(threads >= 64 && threads <= 1024 && threads % 32 == 0,
              "zero_reduce_scatter_bf16: 64..1024 threads, whole warps");
  TORCH_CHECK(seq >= 0 && seq < kSeqPerStep, "zero_reduce_scatter_bf16: launch sequence number out of range");
  const int world = (int)grad_peers.size();
  TORCH_CHECK(seg_lo % 64 == 0 && shard_len % 64 == 0, "zero_reduce_scatter_bf16: 64-element aligned segments");
  TORCH_CHECK(partial.scalar_type() == at::kFloat && partial.is_cuda() && partial.numel() >= 1 &&
                  partial.numel() <= kMaxBlocks,
              "zero_reduce_scatter_bf16: partial sums buffer of 1..", kMaxBlocks, " floats expected");
  TORCH_CHECK(epoch.scalar_type() == at::kInt && epoch.is_cuda(), "zero_reduce_scatter_bf16: int32 device epoch");
  c10::cuda::CUDAGuard guard(partial.device());
  const int grid = (int)partial.numel();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  zero_reduce_scatter_bf16_kernel<<<grid, (int)threads, 0, stream>>>(
      to_peers(grad_peers, world), to_peers(grad16_peers, world), to_peers(flag_peers, world), seg_lo, shard_len,
      partial.data_ptr<float>(), epoch.data_ptr<int>(), (int)rank, world, (int)seq, timeout_from_ms(timeout_ms),
      error_word(partial.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void zero_norm_exchange(std::vector<int64_t> flag_peers, at::Tensor partial, at::Tensor epoch, int64_t rank,
                        double max_norm, at::Tensor grad_scale, at::Tensor grad_norm, double timeout_ms) {
  const int world = (int)flag_peers.size();
  c10::cuda::CUDAGuard guard(partial.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  zero_norm_exchange_kernel<<<1, 32, 0, stream>>>(to_peers(flag_peers, world), partial.data_ptr<float>(),
                                                  (int)partial.numel(), epoch.data_ptr<int>(), (int)rank, world,
                                                  (float)max_norm, grad_scale.data_ptr<float>(),
                                                  grad_norm.data_ptr<float>(), timeout_from_ms(timeout_ms),
                                                  error_word(partial.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void zero_all_gather(std::vector<int64_t> data_peers, std::vector<int64_t> shadow_peers, std::vector<int64_t> flag_peers,
                     int64_t seg_lo, int64_t shard_len, int64_t bf16_begin, at::Tensor epoch, int64_t rank, int64_t blocks,
                     double timeout_ms, int64_t seq) {
  const int world = (int)data_peers.size();
  TORCH_CHECK(seg_lo % 64 == 0 && shard_len % 64 == 0 && bf16_begin % 64 == 0,
              "zero_all_gather: 64-element aligned segments expected");
  TORCH_CHECK(seq >= 0 && seq < kSeqPerStep, "zero_all_gather: launch sequence number out of range");
  TORCH_CHECK(blocks >= 1 && blocks <= kMaxBlocks, "zero_all_gather: 1..", kMaxBlocks, " blocks");
  c10::cuda::CUDAGuard guard(epoch.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  zero_all_gather_kernel<<<(int)blocks, 512, 0, stream>>>(to_peers(data_peers, world), to_peers(shadow_peers, world),
                                                          to_peers(flag_peers, world), seg_lo, shard_len, bf16_begin,
                                                          epoch.data_ptr<int>(), (int)rank, world, (int)seq,
                                                          timeout_from_ms(timeout_ms), error_word(epoch.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void zero_advance_epoch(at::Tensor epoch) {
  c10::cuda::CUDAGuard guard(epoch.device());
  zero_advance_epoch_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(epoch.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
