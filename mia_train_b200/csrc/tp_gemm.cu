// Fused tensor-parallel collective GEMMs over NVLink peer memory (sequence-parallel Megatron layout).
//
// Under sequence parallelism the residual stream stays sharded by token: rank r of W holds rows
// [r S, (r + 1) S) of the (M, C) activations, S = M / W. A column-parallel layer (qkv, fc1, and the
// dX GEMMs of the row-parallel layers in backward) needs every row of its input; a row-parallel
// layer (proj, fc2, and the dX GEMMs of column-parallel layers) produces partial sums over this
// rank's share of the features, which are summed over ranks and scattered back by token. Each of
// the two kernels below does the math and the transfer in one launch:
//
//   tp_ag_gemm   D[M, N] = epi( gather_q(A_q)[M, K] . B[N, K]^T ),  A_r = this rank's (S, K) rows.
//   tp_gemm_rs   O_r[S, N] = epi( sum_q (A_q[M, K] . B_q^T)[rows of rank r] ).
//
// Both are persistent tcgen05 GEMMs (one CTA per SM, warp 0 issues TMA, warp 1 issues
// tcgen05.mma into double-buffered TMEM accumulators, eight epilogue warps drain TMEM). What is
// added:
//
// all-gather -> GEMM. CTA b owns the 128-row blocks b, b + G, ... of the gathered M (G = grid), so
// every row block is fetched exactly once per GPU and no CTA waits on another CTA of its GPU. Four
// copy warps per CTA first copy the CTA's local rows (A_r) into this rank's symmetric send buffer
// and into the gathered output, and publish each block to every peer with a system-scope release
// flag; then they pull the remote rows of their blocks from the peers' send buffers with 16-byte
// loads over NVLink (12 in flight per thread) into the gathered output, 128 columns at a time,
// advancing a shared-memory progress counter. The TMA producer waits on that counter before it
// loads a K slice of a block's first N tile; the other N tiles of the block re-read the rows from
// local memory. Blocks whose rows are all local are computed first, so the tensor cores start
// while the remote rows are still in flight. The gathered A is an output: the backward pass uses
// it for the weight gradient.
//
// GEMM -> reduce-scatter. CTA b owns row blocks b, b + G, ... and computes all N tiles of a block
// in a row, visiting the blocks owned by the next rank first and this rank's own last. The
// epilogue rounds each accumulator row to bf16 and stores it straight into the owner's receive
// slot (peer stores over NVLink, or local stores for this rank's own rows), releases the
// accumulator to the MMA warp, and once the block's last N tile is stored publishes the block to
// its owner(s) with one system fence per warp.
// After its last tile every CTA reduces some of this rank's row blocks: it waits for the block's
// flags from every rank, sums the W slots in fp32 and applies bias, LayerScale and the residual add
// before the single bf16 store.
//
// Buffers and ordering. Send and receive buffers are double-buffered by the parity of a per-kind
// epoch counter kept on the device (advanced by the last CTA of every launch, so a captured CUDA
// graph replays correctly). A rank writes buffer e % 2 in launch e; every peer last read it in
// launch e - 2, and this rank has proof that every peer finished launch e - 2: in launch e - 1 it
// waited for data that each peer published at the start of its launch e - 1. Flags hold the epoch
// of the launch that published, so they only grow. Every rank must issue the same sequence of
// these launches (every TP layer's forward and backward does, on every rank).
//
// Co-residency. CTAs wait on flags that CTAs of other GPUs publish, which in turn may wait on this
// GPU: the kernels are launched cooperatively, so all CTAs of a launch are resident together.
// Every wait is bounded (%globaltimer); on expiry the kernel records an error code in the device
// error word and unwinds (drains its copies and MMAs, frees tensor memory) instead of hanging.
// No load here uses cluster multicast; peers are read and written with plain 16-byte accesses
// only, and TMA reads local memory only.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cstdlib>
#include <vector>

#include "common.cuh"
#include "errors.h"
#include "gemm_common.cuh"

namespace mia {
namespace tp {

constexpr int kMaxWorld = 8;
constexpr int kMaxMBlocks = 2048;  // 128-row blocks of the gathered M: M <= 262144
constexpr int kMaxOwned = 64;      // row blocks per CTA in the all-gather kernel
constexpr int kEpi = 8;            // epilogue warps
constexpr int kAgThreads = 64 + 32 * kEpi + 32;  // producer, MMA, epilogue warps, store warp
constexpr int kRsThreads = 64 + 32 * kEpi;                 // 320

// Flag area of one rank (int32):
//   ag_ready[src][block]  written by src: its rows of gathered block `block` are in its send buffer
//   rs_ready[src][block]  written by src: its partial rows of block `block` are in our receive slot
//   (spare)               kMaxMBlocks ints, unused
//   ctl[]                 local: epochs and exit counters
constexpr int kAgReady = 0;
constexpr int kRsReady = kAgReady + kMaxWorld * kMaxMBlocks;
constexpr int kBlockCount = kRsReady + kMaxWorld * kMaxMBlocks;
constexpr int kCtl = kBlockCount + kMaxMBlocks;
constexpr int kCtlAgEpoch = 0, kCtlAgExit = 1, kCtlRsEpoch = 2, kCtlRsExit = 3;
constexpr int kFlagInts = kCtl + 16;

struct Peers {
  int64_t p[kMaxWorld];
};

__device__ __forceinline__ int64_t pick(const Peers& p, int i) {
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
__device__ __forceinline__ void st_release_cta_shared(int* addr, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(addr)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta_shared(const int* addr) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(addr)) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Bounded wait until *flag >= target (system scope). False on timeout (error recorded).
__device__ __forceinline__ bool wait_flag(const int* flag, int target, uint64_t timeout_ns, volatile int* abort_flag,
                                          int* err, int code) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t start = globaltimer_ns();
  while (ld_acquire_sys(flag) < target) {
    if (abort_flag != nullptr && *abort_flag) return false;
    if (globaltimer_ns() - start > timeout_ns) {
      record_error(err, code);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
  return true;
}

struct TpShape {
  int M, N, K;      // gathered rows, output columns, reduction length
  int S;            // rows per rank (M = S * world)
  int rank, world;
  int num_blocks;   // ceil(M / 128)
};

__device__ __forceinline__ int block_src_lo(const TpShape& s, int mb) { return (mb * 128) / s.S; }
__device__ __forceinline__ int block_src_hi(const TpShape& s, int mb) {
  return (min(mb * 128 + 128, s.M) - 1) / s.S;
}

// ------------------------------------------------------------------------------- all-gather GEMM
// Bounded wait until *counter >= target (shared memory, written by other warps of this CTA).
__device__ __forceinline__ bool spin_ge(const volatile int* counter, int target, volatile int* abort_flag, int* err,
                                        int code) {
  if (*counter >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (*counter < target) {
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > MIA_WAIT_LIMIT_NS) {
      record_error(err, code);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

struct AgParams {
  GemmParams g;                 // M = gathered rows; D, bias, aux, aux_out, act, err
  TpShape s;
  Peers flags;
  uint64_t timeout_ns;
};

// Tensor maps of the all-gather kernel: the gathered output, this rank's rows, and every rank's send
// buffer as a 3-D (K, S, parity) array (index `rank` is this rank's own, used for its stores).
struct AgMaps {
  CUtensorMap full;   // (K, M) gathered A, local
  CUtensorMap local;  // (K, S) this rank's rows, local
  CUtensorMap send[kMaxWorld];
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int BN, int STAGES>
struct AgSmem {
  static constexpr int kBTileBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kBytes = STAGES * kStageBytes + 1024 + 512 + kMaxOwned * 4;
};

// Warp roles: 0 TMA producer, 1 MMA issuer, 2..9 epilogue, 10 store warp (kAgWarps = 11).
//
// CTA b owns the 128-row blocks b, b + G, ... of the gathered M (every block's rows come from one
// rank: S is a multiple of 128 when there are peers). The producer visits this CTA's local blocks
// first, then the remote ones. For every block, the first N tile's K slices of A come by TMA from
// where the rows live -- this rank's own rows, or the owner's send buffer over NVLink -- and the
// store warp writes each such slice, once it has landed in shared memory, to the gathered output
// (and, for local rows, to this rank's send buffer) with TMA stores before it releases the stage;
// the block's other N tiles re-read A from the gathered output. After the last slice of a local
// block is stored, the store warp waits for its stores to complete and publishes the block to every
// peer. The producer waits for a remote block's flag before its first load from the owner.
template <int BN, bool B_MN, int STAGES, int EPI>
__global__ void __launch_bounds__(kAgThreads, 1)
    tp_ag_gemm_kernel(const __grid_constant__ AgMaps maps, const __grid_constant__ CUtensorMap tmB, const AgParams P) {
  using L = AgSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kATileBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* nseq_slot = reinterpret_cast<int*>(tmem_slot + 2);
  int* nlocal_slot = reinterpret_cast<int*>(tmem_slot + 3);
  int* seq = reinterpret_cast<int*>(smem + STAGES * L::kStageBytes + 512);  // owned blocks, compute order

  const GemmParams& p = P.g;
  const TpShape& s = P.s;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr uint32_t kTmemCols = 2 * BN;
  const int num_k = (p.K + kBK - 1) / kBK;
  const int* ctl = reinterpret_cast<const int*>(pick(P.flags, s.rank)) + kCtl;
  const int epoch = *reinterpret_cast<const volatile int*>(ctl + kCtlAgEpoch) + 1;
  const int par = epoch & 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 2);  // the MMA warp's commit and the store warp
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * kEpi);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *reinterpret_cast<volatile int*>(tmem_slot + 4) = 0;
    int n = 0, nl = 0;
    for (int pass = 0; pass < 2; ++pass)
      for (int mb = blockIdx.x; mb < s.num_blocks; mb += gridDim.x) {
        const bool local = block_src_lo(s, mb) == s.rank;
        if ((pass == 0) == local && n < kMaxOwned) {
          seq[n++] = mb;
          nl += local ? 1 : 0;
        }
      }
    *nseq_slot = n;
    *nlocal_slot = nl;
    fence_barrier_init();
    prefetch_tensormap(&maps.full);
    prefetch_tensormap(&maps.local);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nseq = *nseq_slot;
  const int nlocal = *nlocal_slot;
  const int num_n = (p.N + BN - 1) / BN;
  int* my_flags = reinterpret_cast<int*>(pick(P.flags, s.rank));
  volatile int* stored = reinterpret_cast<volatile int*>(tmem_slot + 4);  // first-N-tile slices stored (store warp)
  constexpr int kStoreWarp = 2 + kEpi;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      constexpr uint32_t kTx = kATileBytes + L::kBTileBytes;
      for (int i = 0; i < nseq && ok; ++i) {
        const int mb = seq[i];
        const int m0 = mb * 128;
        const int src = block_src_lo(s, mb);
        const bool local = i < nlocal;
        if (!local) {
          if (!wait_flag(my_flags + kAgReady + src * kMaxMBlocks + mb, epoch, P.timeout_ns, abort_flag, p.err,
                         kErrTpChunkWait)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        for (int nt = 0; nt < num_n && ok; ++nt) {
          const int n0 = nt * BN;
          for (int kb = 0; kb < num_k; ++kb) {
            if (!local && nt > 0 && !spin_ge(stored, i * num_k + kb + 1, abort_flag, p.err, kErrTpChunkWait)) {
              ok = false;
              break;
            }
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrGemmProducerWait)) {
              ok = false;
              break;
            }
            const int k0 = kb * kBK;
            mbar_arrive_expect_tx(&full_bar[stage], kTx);
            uint8_t* a_dst = smA + stage * kATileBytes;
            uint8_t* b_dst = smB + stage * L::kBTileBytes;
            if (local) {
              tma_load_2d(a_dst, &maps.local, &full_bar[stage], k0, m0 - s.rank * s.S);
            } else if (nt == 0) {
              tma_load_3d(a_dst, &maps.send[src], &full_bar[stage], k0, m0 - src * s.S, par);
            } else {
              fence_proxy_async_global();
              tma_load_2d(a_dst, &maps.full, &full_bar[stage], k0, m0);
            }
            if (!B_MN) {
              tma_load_2d(b_dst, &tmB, &full_bar[stage], k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0);
            }
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        int st = stage, ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--st < 0) {
            st = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(&full_bar[st], ph, nullptr, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, false, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, any = false;
      for (int i = 0; i < nseq && ok; ++i) {
        for (int nt = 0; nt < num_n && ok; ++nt) {
          if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.err, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          for (int kb = 0; kb < num_k; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrGemmMmaWait)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smA + stage * kATileBytes);
            const uint32_t b_base = smem_u32(smB + stage * L::kBTileBytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const uint64_t a_desc = make_sdesc_sw128(a_base + k * 32, 16, 1024);
              const uint64_t b_desc = B_MN ? make_sdesc_sw128(b_base + k * 2048, 8192, 1024)
                                           : make_sdesc_sw128(b_base + k * 32, 16, 1024);
              tc_mma_f16(d_tmem, a_desc, b_desc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
              any = true;
            }
            tc_commit(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          tc_commit(&tfull_bar[acc]);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1;
        }
      }
      if (!ok && any) {
        tc_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, nullptr, 0);
      }
    }
  } else if (warp == kStoreWarp) {
    if (lane == 0) {
      // ---------------- store warp: first-N-tile A slices -> gathered output (+ send buffer)
      int stage = 0;
      uint32_t phase = 0;
      int done = 0;
      bool ok = true;
      for (int i = 0; i < nseq && ok; ++i) {
        const int mb = seq[i];
        const int m0 = mb * 128;
        const bool local = i < nlocal;
        for (int nt = 0; nt < num_n && ok; ++nt) {
          for (int kb = 0; kb < num_k; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrTpChunkWait)) {
              ok = false;
              break;
            }
            if (nt == 0) {
              const uint8_t* a_src = smA + stage * kATileBytes;
              tma_store_2d(&maps.full, a_src, kb * kBK, m0);
              if (local && s.world > 1) tma_store_3d(&maps.send[s.rank], a_src, kb * kBK, m0 - s.rank * s.S, par);
              bulk_commit();
              bulk_wait_all();  // written (not only read): the producer may re-read these rows next
              ++done;
              asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)stored)), "r"(done)
                           : "memory");
            }
            mbar_arrive(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (nt == 0 && ok && local && s.world > 1) {
            // every K slice of this local block is in the send buffer: publish it to the peers
            fence_proxy_async_global();
            __threadfence_system();
            for (int q = 0; q < s.world; ++q)
              if (q != s.rank)
                st_release_sys(reinterpret_cast<int*>(pick(P.flags, q)) + kAgReady + s.rank * kMaxMBlocks + mb,
                               epoch);
          }
        }
      }
      bulk_wait_all();
    }
  } else if (warp >= 2 && warp < 2 + kEpi) {
    // ---------------- epilogue warps 2..9
    const int lane_group = warp % 4;
    const int col_part = (warp - 2) / 4;  // two column halves
    constexpr int kPartCols = BN / 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int i = 0; i < nseq && ok; ++i) {
      const int m = seq[i] * 128 + lane_group * 32 + lane;
      for (int nt = 0; nt < num_n; ++nt) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrGemmEpilogueWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int n0 = nt * BN + col_part * kPartCols;
        const uint32_t t_row = tmem_base + ((uint32_t)(lane_group * 32) << 16) + acc * BN + col_part * kPartCols;
#pragma unroll 1
        for (int c = 0; c < kPartCols / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait_regs(r);
          epilogue_chunk<EPI>(p, m, n0 + c * 32, r);
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) {
    int* wctl = my_flags + kCtl;
    __threadfence();
    if (atomicAdd(wctl + kCtlAgExit, 1) == (int)gridDim.x - 1) {
      wctl[kCtlAgExit] = 0;
      __threadfence();
      wctl[kCtlAgEpoch] = epoch;
    }
  }
}

// ------------------------------------------------------------------------- GEMM reduce-scatter
struct RsParams {
  TpShape s;
  int* err;
  Peers recv;        // every rank's receive area: [parity][src][S][N] bf16
  int64_t recv_parity_elems;
  Peers flags;
  // reduce epilogue: out = residual + gamma * (sum + bias); `pre_out` keeps sum + bias
  __nv_bfloat16* out;
  const float* bias;
  const float* gamma;
  const __nv_bfloat16* residual;
  __nv_bfloat16* pre_out;
  uint64_t timeout_ns;
};

template <int BN, int STAGES>
struct RsSmem {
  static constexpr int kBTileBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  // one bf16 output tile, 16-byte chunks XOR-swizzled by row (the staged, 128-column variant only)
  static constexpr int kStagingBytes = BN == 128 ? 128 * BN * 2 : 0;
  static constexpr int kBytes = STAGES * kStageBytes + kStagingBytes + 1024 + 512 + kMaxOwned * 4 + 256;
};



// CTA b owns the 128-row blocks b, b + G, ... and computes every N tile of a block before the next
// block, so it alone decides when a block's partial rows are complete and publishes them. Blocks
// are visited by owner distance: rows of the next rank first, this rank's own rows last.
template <int BN, bool A_MN, bool B_MN, int STAGES>
__global__ void __launch_bounds__(kRsThreads, 1)
    tp_gemm_rs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const RsParams P) {
  using L = RsSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kATileBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* block_arrivals = reinterpret_cast<int*>(tmem_slot + 2);  // [4], by block sequence index mod 4
  int* nseq_slot = reinterpret_cast<int*>(tmem_slot + 6);
  volatile int* staged = reinterpret_cast<volatile int*>(tmem_slot + 7);  // epilogue warps done writing the tile
  volatile int* drained = reinterpret_cast<volatile int*>(tmem_slot + 8);  // ... done storing it out
  int* seq = reinterpret_cast<int*>(smem + STAGES * L::kStageBytes + 512);
  uint4* staging = reinterpret_cast<uint4*>(smem + STAGES * L::kStageBytes + 512 + kMaxOwned * 4);

  const TpShape& s = P.s;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr uint32_t kTmemCols = 2 * BN;
  const int num_k = (s.K + kBK - 1) / kBK;
  const int num_n = (s.N + BN - 1) / BN;
  int* my_flags = reinterpret_cast<int*>(pick(P.flags, s.rank));
  const int epoch = *reinterpret_cast<const volatile int*>(my_flags + kCtl + kCtlRsEpoch) + 1;
  const int64_t par_off = (epoch & 1) ? P.recv_parity_elems : 0;
  const int64_t slot_elems = (int64_t)s.S * s.N;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * kEpi);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    for (int j = 0; j < 4; ++j) block_arrivals[j] = 0;
    *staged = 0;
    *drained = 0;
    int n = 0;
    for (int d = 1; d <= s.world; ++d) {
      const int owner = (s.rank + d) % s.world;
      for (int mb = blockIdx.x; mb < s.num_blocks; mb += gridDim.x)
        if (block_src_lo(s, mb) == owner && n < kMaxOwned) seq[n++] = mb;
    }
    *nseq_slot = n;
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nseq = *nseq_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      constexpr uint32_t kTx = kATileBytes + L::kBTileBytes;
      for (int i = 0; i < nseq && ok; ++i) {
        const int m0 = seq[i] * 128;
        for (int nt = 0; nt < num_n && ok; ++nt) {
          const int n0 = nt * BN;
          for (int kb = 0; kb < num_k; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, P.err, kErrGemmProducerWait)) {
              ok = false;
              break;
            }
            const int k0 = kb * kBK;
            mbar_arrive_expect_tx(&full_bar[stage], kTx);
            uint8_t* a_dst = smA + stage * kATileBytes;
            uint8_t* b_dst = smB + stage * L::kBTileBytes;
            if (!A_MN) {
              tma_load_2d(a_dst, &tmA, &full_bar[stage], k0, m0);
            } else {
#pragma unroll
              for (int j = 0; j < 2; ++j) tma_load_2d(a_dst + j * 8192, &tmA, &full_bar[stage], m0 + 64 * j, k0);
            }
            if (!B_MN) {
              tma_load_2d(b_dst, &tmB, &full_bar[stage], k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0);
            }
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        int st = stage, ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--st < 0) {
            st = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(&full_bar[st], ph, nullptr, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, any = false;
      for (int i = 0; i < nseq && ok; ++i) {
        for (int nt = 0; nt < num_n && ok; ++nt) {
          if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, P.err, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          for (int kb = 0; kb < num_k; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, P.err, kErrGemmMmaWait)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smA + stage * kATileBytes);
            const uint32_t b_base = smem_u32(smB + stage * L::kBTileBytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const uint64_t a_desc = A_MN ? make_sdesc_sw128(a_base + k * 2048, 8192, 1024)
                                           : make_sdesc_sw128(a_base + k * 32, 16, 1024);
              const uint64_t b_desc = B_MN ? make_sdesc_sw128(b_base + k * 2048, 8192, 1024)
                                           : make_sdesc_sw128(b_base + k * 32, 16, 1024);
              tc_mma_f16(d_tmem, a_desc, b_desc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
              any = true;
            }
            tc_commit(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          tc_commit(&tfull_bar[acc]);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1;
        }
      }
      if (!ok && any) {
        tc_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, nullptr, 0);
      }
    }
  } else {
    // ---------------- epilogue warps: partial rows -> owner's receive slot
    // BN = 128 (staged): each warp converts its 32 rows x 64 columns to bf16 into the shared staging
    // tile and releases the accumulator; once all eight warps have staged the tile, warp w stores
    // rows [16 w, 16 w + 16) out, two rows of 256 contiguous bytes per instruction, so NVLink writes
    // go out as whole row segments. BN = 256 (direct): each thread stores its own row's 64-byte
    // pieces straight from registers (fewer, wider tiles; better when the stores stay local).
    const int lane_group = warp % 4;
    const int col_part = (warp - 2) / 4;
    const int ew = warp - 2;
    constexpr int kPartCols = BN / 2;
    constexpr int kChunksPerRow = BN / 8;
    const int et = threadIdx.x - 64;  // 0 .. 32 * kEpi - 1
    int acc = 0;
    uint32_t acc_phase = 0;
    int tile_seq = 0;
    bool ok = true;
    for (int i = 0; i < nseq && ok; ++i) {
      const int mb = seq[i];
      __nv_bfloat16* dst_row = nullptr;  // direct variant: this thread's row in its owner's slot
      if constexpr (BN != 128) {
        const int m = mb * 128 + lane_group * 32 + lane;
        if (m < s.M) {
          const int owner = m / s.S;
          dst_row = reinterpret_cast<__nv_bfloat16*>(pick(P.recv, owner)) + par_off + (int64_t)s.rank * slot_elems +
                    (int64_t)(m - owner * s.S) * s.N;
        }
      }
      for (int nt = 0; nt < num_n; ++nt) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, P.err, kErrGemmEpilogueWait) ||
            (BN == 128 && !spin_ge(drained, kEpi * tile_seq, abort_flag, P.err, kErrGemmEpilogueWait))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int n0 = nt * BN;
        const int row = lane_group * 32 + lane;
        const uint32_t t_row = tmem_base + ((uint32_t)(lane_group * 32) << 16) + acc * BN + col_part * kPartCols;
#pragma unroll 1
        for (int c = 0; c < kPartCols / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait_regs(r);
          uint4 packed[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            packed[q] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1])),
                                   pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                                   pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                                   pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
          if constexpr (BN == 128) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int chunk = col_part * (kPartCols / 8) + c * 4 + q;
              staging[row * kChunksPerRow + (chunk ^ (row & 15))] = packed[q];
            }
          } else {
            const int n = n0 + col_part * kPartCols + c * 32;
            if (dst_row != nullptr && n < s.N) {
              if (n + 32 <= s.N) {
#pragma unroll
                for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(dst_row + n)[q] = packed[q];
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (n + j < s.N) dst_row[n + j] = __float2bfloat16_rn(__uint_as_float(r[j]));
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);  // the MMA may refill this accumulator while we store
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        if constexpr (BN == 128) {
          __threadfence_block();
          __syncwarp();
          if (lane == 0) atomicAdd(const_cast<int*>(staged), 1);
          if (!spin_ge(staged, kEpi * (tile_seq + 1), abort_flag, P.err, kErrGemmEpilogueWait)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int tr = 16 * ew + 2 * it + (lane >> 4);
            const int ch = lane & 15;
            const int gm = mb * 128 + tr;
            const int gn = n0 + ch * 8;
            if (gm < s.M && gn < s.N) {
              const int owner = gm / s.S;
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(pick(P.recv, owner)) + par_off +
                                   (int64_t)s.rank * slot_elems + (int64_t)(gm - owner * s.S) * s.N + gn;
              *reinterpret_cast<uint4*>(dst) = staging[tr * kChunksPerRow + (ch ^ (tr & 15))];
            }
          }
          __syncwarp();
          if (lane == 0) atomicAdd(const_cast<int*>(drained), 1);
        }
        ++tile_seq;
      }
      if (!ok) break;
      // The block's partial rows are stored: make them visible system-wide, then the last warp of this
      // CTA publishes the block to its owner(s). A warp is at most two blocks ahead of the slowest
      // one (it needs every warp's release of the accumulator it reuses), so four counters suffice.
      __threadfence_system();
      __syncwarp();
      if (lane == 0 && atomicAdd(&block_arrivals[i & 3], 1) == kEpi - 1) {
        block_arrivals[i & 3] = 0;
        __threadfence_system();
        const int lo = block_src_lo(s, mb), hi = block_src_hi(s, mb);
        for (int q = lo; q <= hi; ++q)
          st_release_sys(reinterpret_cast<int*>(pick(P.flags, q)) + kRsReady + s.rank * kMaxMBlocks + mb, epoch);
      }
    }
    // ---------------- reduce this rank's row blocks (sum of W slots + epilogue)
    if (ok) {
      const int row_lo = s.rank * s.S, row_hi = row_lo + s.S;
      const int mb_lo = row_lo / 128, mb_hi = (row_hi - 1) / 128;
      const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(pick(P.recv, s.rank)) + par_off;
      const int vpr = s.N / 8;
      for (int mb = mb_lo + (int)blockIdx.x; mb <= mb_hi; mb += gridDim.x) {
        // Every thread waits for the block's W slots itself (no barrier that a failed wait could strand).
        bool ready = true;
        for (int q = 0; q < s.world && ready; ++q)
          ready = wait_flag(my_flags + kRsReady + q * kMaxMBlocks + mb, epoch, P.timeout_ns, abort_flag, P.err,
                            kErrTpSlotWait);
        if (!ready) break;
        const int r0 = max(mb * 128, row_lo) - row_lo, r1 = min(mb * 128 + 128, row_hi) - row_lo;
        const int total = (r1 - r0) * vpr;
        // Four 8-element vectors per thread per pass, their W slot loads issued together.
        constexpr int kU = 4;
        constexpr int kStride = 32 * kEpi;
        for (int base = 0; base < total; base += kStride * kU) {
          float a[kU][8];
          int64_t off[kU];
          bool live[kU];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int v = base + u * kStride + et;
            live[u] = v < total;
            const int vv = live[u] ? v : 0;
            off[u] = (int64_t)(r0 + vv / vpr) * s.N + (vv % vpr) * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) a[u][j] = 0.f;
          }
          for (int q = 0; q < s.world; ++q) {
            uint4 x[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u)
              if (live[u]) x[u] = __ldcg(reinterpret_cast<const uint4*>(recv + q * slot_elems + off[u]));
#pragma unroll
            for (int u = 0; u < kU; ++u) {
              if (!live[u]) continue;
              const uint32_t w[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                a[u][2 * h] += bf16_lo(w[h]);
                a[u][2 * h + 1] += bf16_hi(w[h]);
              }
            }
          }
          uint4 res[kU];
          if (P.residual != nullptr) {
#pragma unroll
            for (int u = 0; u < kU; ++u)
              if (live[u]) res[u] = __ldg(reinterpret_cast<const uint4*>(P.residual + off[u]));
          }
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            if (!live[u]) continue;
            const int n = (int)(off[u] % s.N);
            float* av = a[u];
            if (P.bias != nullptr) {
              const float4 b0 = __ldg(reinterpret_cast<const float4*>(P.bias + n));
              const float4 b1 = __ldg(reinterpret_cast<const float4*>(P.bias + n + 4));
              av[0] += b0.x; av[1] += b0.y; av[2] += b0.z; av[3] += b0.w;
              av[4] += b1.x; av[5] += b1.y; av[6] += b1.z; av[7] += b1.w;
            }
            if (P.pre_out != nullptr)
              *reinterpret_cast<uint4*>(P.pre_out + off[u]) = make_uint4(
                  pack_bf16x2(av[0], av[1]), pack_bf16x2(av[2], av[3]), pack_bf16x2(av[4], av[5]), pack_bf16x2(av[6], av[7]));
            if (P.gamma != nullptr) {
              const float4 g0 = __ldg(reinterpret_cast<const float4*>(P.gamma + n));
              const float4 g1 = __ldg(reinterpret_cast<const float4*>(P.gamma + n + 4));
              av[0] *= g0.x; av[1] *= g0.y; av[2] *= g0.z; av[3] *= g0.w;
              av[4] *= g1.x; av[5] *= g1.y; av[6] *= g1.z; av[7] *= g1.w;
            }
            if (P.residual != nullptr) {
              const uint32_t w[4] = {res[u].x, res[u].y, res[u].z, res[u].w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                av[2 * h] += bf16_lo(w[h]);
                av[2 * h + 1] += bf16_hi(w[h]);
              }
            }
            *reinterpret_cast<uint4*>(P.out + off[u]) = make_uint4(
                pack_bf16x2(av[0], av[1]), pack_bf16x2(av[2], av[3]), pack_bf16x2(av[4], av[5]), pack_bf16x2(av[6], av[7]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(my_flags + kCtl + kCtlRsExit, 1) == (int)gridDim.x - 1) {
      my_flags[kCtl + kCtlRsExit] = 0;
      __threadfence();
      my_flags[kCtl + kCtlRsEpoch] = epoch;
    }
  }
}

// ---------------------------------------------------------------------------------------- host
Peers to_peers(const std::vector<int64_t>& v, int world, const char* what) {
  TORCH_CHECK((int)v.size() == world && world >= 1 && world <= kMaxWorld, what, ": expected ", world,
              " peer pointers (world 1..", kMaxWorld, ")");
  Peers p{};
  for (int i = 0; i < world; ++i) {
    TORCH_CHECK(v[i] != 0 && (v[i] & 255) == 0, what, ": peer pointers must be non-null and 256-byte aligned");
    p.p[i] = v[i];
  }
  return p;
}

template <typename Kern, typename... Args>
void coop_launch(Kern kern, int grid, int threads, int smem_bytes, cudaStream_t stream, const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, args...));
}

int64_t flag_bytes() { return (int64_t)kFlagInts * 4; }

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int BN, bool B_MN, int EPI>
static void launch_ag(const AgMaps& maps, const CUtensorMap& tb, const AgParams& prm, int grid, cudaStream_t st,
                      int device) {
  constexpr int ST = BN == 256 ? 4 : 6;
  using L = AgSmem<BN, ST>;
  auto kern = tp_ag_gemm_kernel<BN, B_MN, ST, EPI>;
  static bool configured[64] = {false};
  if (!configured[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[device] = true;
  }
  coop_launch(kern, grid, kAgThreads, L::kBytes, st, maps, tb, prm);
}

template <int BN, bool B_MN>
static void dispatch_ag_epi(int epi, const AgMaps& maps, const CUtensorMap& tb, const AgParams& prm, int grid,
                            cudaStream_t st, int device) {
  if (epi == kEpiGelu) launch_ag<BN, B_MN, kEpiGelu>(maps, tb, prm, grid, st, device);
  else if (epi == kEpiDGelu) launch_ag<BN, B_MN, kEpiDGelu>(maps, tb, prm, grid, st, device);
  else launch_ag<BN, B_MN, kEpiPlain>(maps, tb, prm, grid, st, device);
}

// (K, S, 2) bf16 tensor map over a send area: rows of K elements, two parities `parity_bytes` apart.
static CUtensorMap send_map(int64_t base, int64_t K, int64_t S, int64_t parity_bytes) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)S, 2};
  cuuint64_t strides[2] = {(cuuint64_t)(K * 2), (cuuint64_t)parity_bytes};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, reinterpret_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (send buffer) failed with ", (int)r);
  return map;
}

}  // namespace tp

// D = epi(gather(A) . B^T). a_local (S, K) bf16 this rank's rows; b (N, K) (b_kmajor) or (K, N);
// out (M, N) bf16; a_full (M, K) bf16 receives the gathered A. `send_peers[q]` is rank q's send area
// (two parities of `send_parity_bytes` each), `flag_peers[q]` its flag area.
void tp_ag_gemm(at::Tensor a_local, at::Tensor b, at::Tensor out, at::Tensor a_full, c10::optional<at::Tensor> bias,
                c10::optional<at::Tensor> aux, c10::optional<at::Tensor> aux_out, bool b_kmajor, int64_t act,
                std::vector<int64_t> flag_peers, std::vector<int64_t> send_peers, int64_t send_parity_bytes,
                int64_t rank, double timeout_ms) {
  using namespace tp;
  const int world = (int)flag_peers.size();
  TORCH_CHECK(a_local.is_cuda() && a_local.scalar_type() == at::kBFloat16 && a_local.dim() == 2 &&
                  a_local.is_contiguous(),
              "tp_ag_gemm: a_local must be a contiguous bf16 (S, K) CUDA matrix");
  const int64_t S = a_local.size(0), K = a_local.size(1), M = S * world;
  TORCH_CHECK(b.scalar_type() == at::kBFloat16 && b.dim() == 2 && b.is_contiguous(), "tp_ag_gemm: bf16 B expected");
  const int64_t N = b_kmajor ? b.size(0) : b.size(1);
  TORCH_CHECK((b_kmajor ? b.size(1) : b.size(0)) == K, "tp_ag_gemm: K mismatch");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == M && out.size(1) == N,
              "tp_ag_gemm: out must be a contiguous bf16 (M, N) matrix");
  TORCH_CHECK(a_full.scalar_type() == at::kBFloat16 && a_full.is_contiguous() && a_full.size(0) == M &&
                  a_full.size(1) == K,
              "tp_ag_gemm: a_full must be a contiguous bf16 (M, K) matrix");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0 && S >= 1, "tp_ag_gemm: K and N must be multiples of 8");
  TORCH_CHECK((M + 127) / 128 <= kMaxMBlocks, "tp_ag_gemm: at most ", kMaxMBlocks * 128, " gathered rows");
  TORCH_CHECK(S * K * 2 <= send_parity_bytes, "tp_ag_gemm: send buffer too small (", send_parity_bytes, " bytes for ",
              S * K * 2, ")");
  TORCH_CHECK(send_parity_bytes % 256 == 0, "tp_ag_gemm: send parity stride must be a multiple of 256 bytes");
  TORCH_CHECK(al16(a_local.data_ptr()) && al16(b.data_ptr()) && al16(out.data_ptr()) && al16(a_full.data_ptr()),
              "tp_ag_gemm: 16-byte aligned operands expected");
  TORCH_CHECK(rank >= 0 && rank < world, "tp_ag_gemm: rank out of range");
  TORCH_CHECK(world == 1 || S % 128 == 0,
              "tp_ag_gemm: with peers, every rank's row count must be a multiple of 128 (pad the tokens)");
  TORCH_CHECK(act != kActDGelu || aux.has_value(), "tp_ag_gemm: GELU' needs aux");
  c10::cuda::CUDAGuard guard(a_local.device());
  const int device = a_local.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  AgParams prm{};
  GemmParams& p = prm.g;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.D = out.data_ptr();
  p.act = (int)act;
  p.splits = 1;
  p.err = error_word(device);
  auto vec = [&](const c10::optional<at::Tensor>& t) -> const float* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == N,
                "tp_ag_gemm: bias must be a contiguous fp32 vector of length N");
    return t->data_ptr<float>();
  };
  auto mat = [&](const c10::optional<at::Tensor>& t) -> __nv_bfloat16* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->size(0) == M && t->size(1) == N &&
                    al16(t->data_ptr()),
                "tp_ag_gemm: aux tensors must be contiguous bf16 (M, N) matrices");
    return reinterpret_cast<__nv_bfloat16*>(t->data_ptr());
  };
  p.bias = vec(bias);
  p.aux = mat(aux);
  p.aux_out = mat(aux_out);
  prm.s = TpShape{(int)M, (int)N, (int)K, (int)S, (int)rank, world, (int)((M + 127) / 128)};
  prm.flags = to_peers(flag_peers, world, "tp_ag_gemm flags");
  prm.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms * 1e6 : 5e9);

  const int grid = (int)std::min<int64_t>(prm.s.num_blocks, sm_count(device));
  TORCH_CHECK(prm.s.num_blocks <= (int64_t)grid * kMaxOwned, "tp_ag_gemm: too many row blocks per CTA");
  const int bn = N <= 128 ? 128 : 256;
  const int epi = act == kActGelu ? kEpiGelu : (act == kActDGelu ? kEpiDGelu : kEpiPlain);
  AgMaps maps{};
  maps.full = make_bf16_map(a_full.data_ptr(), K, M, K, 64, kBM);
  maps.local = make_bf16_map(a_local.data_ptr(), K, S, K, 64, kBM);
  const Peers send = to_peers(send_peers, world, "tp_ag_gemm send");
  for (int q = 0; q < world; ++q) maps.send[q] = send_map(send.p[q], K, S, send_parity_bytes);
  CUtensorMap tb = b_kmajor ? make_bf16_map(b.data_ptr(), K, N, K, 64, bn) : make_bf16_map(b.data_ptr(), N, K, N, 64, 64);
  if (bn == 256) {
    if (b_kmajor) dispatch_ag_epi<256, false>(epi, maps, tb, prm, grid, stream, device);
    else dispatch_ag_epi<256, true>(epi, maps, tb, prm, grid, stream, device);
  } else {
    if (b_kmajor) dispatch_ag_epi<128, false>(epi, maps, tb, prm, grid, stream, device);
    else dispatch_ag_epi<128, true>(epi, maps, tb, prm, grid, stream, device);
  }
}

namespace tp {
template <int BN, bool A_MN, bool B_MN>
static void launch_rs(const CUtensorMap& ta, const CUtensorMap& tb, const RsParams& prm, int grid, cudaStream_t st,
                      int device) {
  constexpr int ST = BN == 128 ? 5 : 4;
  using L = RsSmem<BN, ST>;
  auto kern = tp_gemm_rs_kernel<BN, A_MN, B_MN, ST>;
  static bool configured[64] = {false};
  if (!configured[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[device] = true;
  }
  coop_launch(kern, grid, kRsThreads, L::kBytes, st, ta, tb, prm);
}
}  // namespace tp

// O_r = residual + gamma * (sum_q (A_q . B_q^T)[rows of r] + bias). a (M, K) bf16 (K-major) holds
// every row of this rank's partial product input; b (N, K) (b_kmajor) or (K, N); out (S, N) bf16
// with S = M / world. `recv_peers[q]` is rank q's receive area (two parities of
// `recv_parity_bytes`, each holding world slots of S x N bf16). `pre_out` (S, N) keeps sum + bias.
void tp_gemm_rs(at::Tensor a, at::Tensor b, at::Tensor out, c10::optional<at::Tensor> bias,
                c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> residual,
                c10::optional<at::Tensor> pre_out, bool b_kmajor, std::vector<int64_t> flag_peers,
                std::vector<int64_t> recv_peers, int64_t recv_parity_bytes, int64_t rank, double timeout_ms) {
  using namespace tp;
  const int world = (int)flag_peers.size();
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.dim() == 2 && a.is_contiguous(),
              "tp_gemm_rs: a must be a contiguous bf16 (M, K) CUDA matrix");
  const int64_t M = a.size(0), K = a.size(1);
  TORCH_CHECK(M % world == 0, "tp_gemm_rs: M must be divisible by the world size");
  const int64_t S = M / world;
  TORCH_CHECK(b.scalar_type() == at::kBFloat16 && b.dim() == 2 && b.is_contiguous(), "tp_gemm_rs: bf16 B expected");
  const int64_t N = b_kmajor ? b.size(0) : b.size(1);
  TORCH_CHECK((b_kmajor ? b.size(1) : b.size(0)) == K, "tp_gemm_rs: K mismatch");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == S && out.size(1) == N,
              "tp_gemm_rs: out must be a contiguous bf16 (M / world, N) matrix");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "tp_gemm_rs: K and N must be multiples of 8");
  TORCH_CHECK((M + 127) / 128 <= kMaxMBlocks, "tp_gemm_rs: at most ", kMaxMBlocks * 128, " rows");
  TORCH_CHECK((int64_t)world * S * N * 2 <= recv_parity_bytes && recv_parity_bytes % 256 == 0,
              "tp_gemm_rs: receive buffer too small or misaligned");
  TORCH_CHECK(al16(a.data_ptr()) && al16(b.data_ptr()) && al16(out.data_ptr()), "tp_gemm_rs: 16-byte aligned operands");
  TORCH_CHECK(rank >= 0 && rank < world, "tp_gemm_rs: rank out of range");
  c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  RsParams prm{};
  prm.s = TpShape{(int)M, (int)N, (int)K, (int)S, (int)rank, world, (int)((M + 127) / 128)};
  prm.err = error_word(device);
  prm.recv = to_peers(recv_peers, world, "tp_gemm_rs recv");
  prm.recv_parity_elems = recv_parity_bytes / 2;
  prm.flags = to_peers(flag_peers, world, "tp_gemm_rs flags");
  prm.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto vec = [&](const c10::optional<at::Tensor>& t) -> const float* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == N,
                "tp_gemm_rs: bias / gamma must be contiguous fp32 vectors of length N");
    return t->data_ptr<float>();
  };
  auto mat = [&](const c10::optional<at::Tensor>& t) -> __nv_bfloat16* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->size(0) == S && t->size(1) == N &&
                    al16(t->data_ptr()),
                "tp_gemm_rs: residual / pre_out must be contiguous bf16 (M / world, N) matrices");
    return reinterpret_cast<__nv_bfloat16*>(t->data_ptr());
  };
  prm.bias = vec(bias);
  prm.gamma = vec(gamma);
  prm.residual = mat(residual);
  prm.pre_out = mat(pre_out);
  prm.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms * 1e6 : 5e9);
  // 128-column tiles with the shared-memory staged epilogue when partial rows cross NVLink, 256-column
  // tiles storing straight from registers for one rank (MIA_TP_RS_STAGED=0|1 overrides).
  static const int staged_env = [] {
    const char* v = std::getenv("MIA_TP_RS_STAGED");
    return v == nullptr ? -1 : std::atoi(v);
  }();
  const bool staged = staged_env >= 0 ? staged_env != 0 : world > 1;
  const int bn = staged || N <= 128 ? 128 : 256;
  const int grid = (int)std::min<int64_t>(prm.s.num_blocks, sm_count(device));
  TORCH_CHECK(prm.s.num_blocks <= (int64_t)grid * kMaxOwned, "tp_gemm_rs: too many row blocks per CTA");
  CUtensorMap ta = make_bf16_map(a.data_ptr(), K, M, K, 64, kBM);
  CUtensorMap tb = b_kmajor ? make_bf16_map(b.data_ptr(), K, N, K, 64, bn) : make_bf16_map(b.data_ptr(), N, K, N, 64, 64);
  if (bn == 128) {
    if (b_kmajor) launch_rs<128, false, false>(ta, tb, prm, grid, stream, device);
    else launch_rs<128, false, true>(ta, tb, prm, grid, stream, device);
  } else {
    if (b_kmajor) launch_rs<256, false, false>(ta, tb, prm, grid, stream, device);
    else launch_rs<256, false, true>(ta, tb, prm, grid, stream, device);
  }
}

int64_t tp_flag_bytes() { return tp::flag_bytes(); }

}  // namespace mia
