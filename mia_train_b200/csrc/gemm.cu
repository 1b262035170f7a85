// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), persistent and warp-specialised.
//
//   D[M, N] = epilogue( sum_k A[m, k] * B[n, k] )
//
// A is read K-major (row-major M x K) or M-major (row-major K x M); B K-major (N x K) or N-major
// (K x N). The transposed reads serve the backward pass: dX = dY W reads W N-major and
// dW = dY^T X reads both operands M/N-major, so no transpose is ever materialised.
//
// CTA = 2 + kEpiWarps warps, one CTA per SM, persistent over output tiles of 128 x BN:
//   warp 0      TMA producer: one thread streams 128x64 A and BNx64 B tiles (128-byte swizzle)
//               into a STAGES-deep shared-memory ring, one mbarrier per stage.
//   warp 1      MMA issuer: allocates 2*BN TMEM columns (two fp32 accumulators), one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) per 16-wide K slice and commits each consumed stage
//               back to the producer and each finished tile to the epilogue.
//   warps 2..   epilogue (kEpiWarps of them): tcgen05.ld of the accumulator (warp w owns TMEM
//               lanes 32*(w%4)..+31, i.e. output rows; each group of four warps takes one part of
//               the tile's columns), bias / GELU (keeping the pre-activation) / GELU' / LayerScale / residual /
//               accumulate-into-output, then 16-byte stores. Latency is hidden across the epilogue
//               warps. While the epilogue drains one accumulator the MMA warp fills the other.
//
// All waits are bounded (see common.cuh); on a timeout the kernel records an error code, drains
// the copies and MMAs it issued, frees its tensor memory and returns.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "errors.h"
#include "gemm_common.cuh"

namespace mia {

template <int BN, bool A_MN, bool B_MN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                        const GemmParams p) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kATileBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;      // [2]
  uint64_t* drain_bar = tempty_bar + 2;      // [1]
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  constexpr uint32_t kTmemCols = 2 * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int num_k = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      constexpr uint32_t kTx = kATileBytes + L::kBTileBytes;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const TileCoord tc = tile_coord(p, tile, BN, num_k);
        const int m0 = tc.m0, n0 = tc.n0;
        for (int kb = tc.kb_begin; kb < tc.kb_end; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrGemmProducerWait)) {
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
            for (int j = 0; j < kBM / 64; ++j) tma_load_2d(a_dst + j * 8192, &tmA, &full_bar[stage], m0 + 64 * j, k0);
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
        if constexpr (!A_MN && !B_MN) {
          const int num_k2 = (p.K2 + kBK - 1) / kBK;
          for (int kb = 0; kb < num_k2 && ok; ++kb) {  // the second operand pair, same accumulator
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrGemmProducerWait)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full_bar[stage], kTx);
            tma_load_2d(smA + stage * kATileBytes, &tmA2, &full_bar[stage], kb * kBK, m0);
            tma_load_2d(smB + stage * L::kBTileBytes, &tmB2, &full_bar[stage], kb * kBK, n0);
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        // Let the copies already in flight land before this CTA's shared memory goes away.
        int s = stage, ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(&full_bar[s], ph, nullptr, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool any_mma = false;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.err, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const TileCoord tc = tile_coord(p, tile, BN, num_k);
        for (int kb = tc.kb_begin; kb < tc.kb_end; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrGemmMmaWait)) {
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
            tc_mma_f16(d_tmem, a_desc, b_desc, idesc, (kb > tc.kb_begin || k > 0) ? 1u : 0u);
            any_mma = true;
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if constexpr (!A_MN && !B_MN) {
          const int num_k2 = (p.K2 + kBK - 1) / kBK;
          for (int kb = 0; kb < num_k2 && ok; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrGemmMmaWait)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smA + stage * kATileBytes);
            const uint32_t b_base = smem_u32(smB + stage * L::kBTileBytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              tc_mma_f16(d_tmem, make_sdesc_sw128(a_base + k * 32, 16, 1024), make_sdesc_sw128(b_base + k * 32, 16, 1024),
                         idesc, 1u);
            tc_commit(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (!ok && any_mma) {
        // Wait for every MMA this thread issued before the tensor memory is released.
        tc_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, nullptr, 0);
      }
    }
  } else {
    // ---------------- epilogue warps 2..9
    const int lane_group = warp % 4;         // TMEM lanes 32*lane_group .. +31
    const int col_part = (warp - 2) / 4;     // which part of the tile's columns
    constexpr int kPartCols = BN / kColParts;
    constexpr int kChunks = kPartCols / 32;  // 32-column chunks per part
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const TileCoord tc = tile_coord(p, tile, BN, (p.K + kBK - 1) / kBK);
      const int m0 = tc.m0;
      const int n0 = tc.n0 + col_part * kPartCols;
      const int m = m0 + lane_group * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(lane_group * 32) << 16) + acc * BN + col_part * kPartCols;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait_regs(r);
        epilogue_chunk<kEpiAll>(p, m, n0 + c * 32, r);
        if (p.colsum != nullptr) colsum_exp_chunk(p, m, n0 + c * 32, r, lane);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------- CTA-pair variant
// Cluster of two CTAs per 256 x BN output tile (cta_group::2). CTA r of the pair loads rows
// m0 + 128 r .. +127 of A and rows n0 + (BN/2) r .. of B into its own shared memory; both sets of
// loads complete on the even CTA's full barrier, whose producer announces the bytes of both. The
// even CTA's MMA warp issues M=256 MMAs that read A and B from both CTAs and write each CTA's 128
// accumulator rows into that CTA's TMEM; its commits arrive on the empty / accumulator-full
// barriers of both CTAs. Both CTAs' epilogue warps release an accumulator on the even CTA's
// accumulator-empty barrier. Per CTA and K block the pair moves 16 KB of A and BN * 64 bytes of B,
// a third less than the single-CTA kernel at BN = 256, for the same tensor work.
template <int BN, int STAGES>
struct PairSmem {
  static constexpr int kBHalfBytes = (BN / 2) * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBHalfBytes;
  static constexpr int kBytes = STAGES * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ TileCoord pair_tile_coord(const GemmParams& p, int tile, int bn, int num_k) {
  const int mn = tile % (p.num_m_tiles * p.num_n_tiles);
  const int split = tile / (p.num_m_tiles * p.num_n_tiles);
  TileCoord c;
  c.m0 = (mn % p.num_m_tiles) * 256;
  c.n0 = (mn / p.num_m_tiles) * bn;
  c.kb_begin = split * p.k_blocks_per_split;
  c.kb_end = min(num_k, c.kb_begin + p.k_blocks_per_split);
  return c;
}

template <int BN, bool A_MN, bool B_MN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const GemmParams p) {
  using L = PairSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kATileBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;      // [2]
  uint64_t* drain_bar = tempty_bar + 2;      // [1]
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x / 2;
  const int num_pairs = gridDim.x / 2;
  constexpr uint32_t kTmemCols = 2 * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // the even CTA's producer; bytes of both CTAs
      mbar_init(&empty_bar[s], 1);  // one commit from the even CTA's MMA warp
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);  // every epilogue warp of both CTAs (even CTA only)
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM of both allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int num_k = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs, own half of A and B)
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      constexpr uint32_t kTxPair = 2 * (kATileBytes + L::kBHalfBytes);
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
        const TileCoord tc = pair_tile_coord(p, tile, BN, num_k);
        const int m0 = tc.m0 + 128 * (int)rank;
        const int n0 = tc.n0 + (BN / 2) * (int)rank;
        for (int kb = tc.kb_begin; kb < tc.kb_end; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          const int k0 = kb * kBK;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], kTxPair);
          uint8_t* a_dst = smA + stage * kATileBytes;
          uint8_t* b_dst = smB + stage * L::kBHalfBytes;
          if (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, &full_bar[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < 2; ++j) tma_load_2d_pair(a_dst + j * 8192, &tmA, &full_bar[stage], m0 + 64 * j, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, &full_bar[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d_pair(b_dst + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && leader) {
        int s = stage, ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(&full_bar[s], ph, nullptr, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (even CTA only)
      constexpr uint32_t idesc = make_idesc_bf16(256, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool any_mma = false;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.err, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const TileCoord tc = pair_tile_coord(p, tile, BN, num_k);
        for (int kb = tc.kb_begin; kb < tc.kb_end; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * kATileBytes);
          const uint32_t b_base = smem_u32(smB + stage * L::kBHalfBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t a_desc = A_MN ? make_sdesc_sw128(a_base + k * 2048, 8192, 1024)
                                         : make_sdesc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t b_desc = B_MN ? make_sdesc_sw128(b_base + k * 2048, 8192, 1024)
                                         : make_sdesc_sw128(b_base + k * 32, 16, 1024);
            tc_mma_f16_pair(d_tmem, a_desc, b_desc, idesc, (kb > tc.kb_begin || k > 0) ? 1u : 0u);
            any_mma = true;
          }
          tc_commit_pair_both(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair_both(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (!ok && any_mma) {
        tc_commit_pair_both(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, nullptr, 0);
      }
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs, own 128 rows)
    const int lane_group = warp % 4;
    const int col_part = (warp - 2) / 4;
    constexpr int kPartCols = BN / kColParts;
    constexpr int kChunks = kPartCols / 32;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < p.num_tiles; tile += num_pairs) {
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const TileCoord tc = pair_tile_coord(p, tile, BN, num_k);
      const int m = tc.m0 + 128 * (int)rank + lane_group * 32 + lane;
      const int n0 = tc.n0 + col_part * kPartCols;
      const uint32_t t_row = tmem_base + ((uint32_t)(lane_group * 32) << 16) + acc * BN + col_part * kPartCols;
      // With kEpiWarps warps per CTA the TMEM and side-input latencies are hidden across warps, so
      // each warp keeps one chunk in flight: its accumulator columns and, loaded while the TMEM
      // load is pending, the side input (GELU' pre-activation or residual).
      const __nv_bfloat16* side = EPI == kEpiDGelu ? p.aux : (EPI == kEpiPlain ? p.residual : nullptr);
      const bool side_ok = side != nullptr && m < p.M && n0 + kChunks * 32 <= p.N;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        uint4 sbuf[4] = {};
        if (side_ok) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            sbuf[q] = __ldg(reinterpret_cast<const uint4*>(side + (size_t)m * p.N + n0 + c * 32) + q);
        }
        tmem_ld_wait_regs(r);
        epilogue_chunk<EPI>(p, m, n0 + c * 32, r, side_ok, sbuf);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&tempty_bar[acc], 0);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer no longer reads this CTA's shared memory or signals its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------ host

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major (rows x inner) matrix with row stride `ld` elements.
static CUtensorMap make_map(const void* base, int64_t inner, int64_t rows, int64_t ld, int box_inner, int box_rows) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", (int)r);
  return map;
}

static int num_sms(int device);

CUtensorMap make_bf16_map(const void* base, int64_t inner, int64_t rows, int64_t ld, int box_inner, int box_rows) {
  return make_map(base, inner, rows, ld, box_inner, box_rows);
}

int sm_count(int device) { return num_sms(device); }

static int num_sms(int device) {
  static int cache[64] = {0};
  if (cache[device] == 0) {
    int v = 0;
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device));
    cache[device] = v;
  }
  return cache[device];
}

template <int BN, bool A_MN, bool B_MN, int STAGES>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2, const CUtensorMap& tb2,
                        GemmParams& p, int device, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, STAGES>;
  static bool configured[64] = {false};
  if (!configured[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[device] = true;
  }
  p.num_m_tiles = (p.M + kBM - 1) / kBM;
  p.num_n_tiles = (p.N + BN - 1) / BN;
  const int num_k = (p.K + kBK - 1) / kBK;
  if (p.splits < 1) p.splits = 1;
  p.k_blocks_per_split = (num_k + p.splits - 1) / p.splits;
  p.splits = (num_k + p.k_blocks_per_split - 1) / p.k_blocks_per_split;  // no empty split
  p.num_tiles = p.num_m_tiles * p.num_n_tiles * p.splits;
  if (p.splits > 1 && !p.accumulate)
    C10_CUDA_CHECK(cudaMemsetAsync(p.D, 0, (size_t)p.M * p.N * sizeof(float), stream));
  const int grid = std::min(p.num_tiles, num_sms(device));
  kern<<<grid, kThreads, L::kBytes, stream>>>(ta, tb, ta2, tb2, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN>
static void dispatch_majors(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2,
                            const CUtensorMap& tb2, GemmParams& p, int device, cudaStream_t s) {
  constexpr int ST = BN == 256 ? 4 : 6;
  if (!a_mn && !b_mn) launch_gemm<BN, false, false, ST>(ta, tb, ta2, tb2, p, device, s);
  else if (!a_mn && b_mn) launch_gemm<BN, false, true, ST>(ta, tb, ta2, tb2, p, device, s);
  else if (a_mn && !b_mn) launch_gemm<BN, true, false, ST>(ta, tb, ta2, tb2, p, device, s);
  else launch_gemm<BN, true, true, ST>(ta, tb, ta2, tb2, p, device, s);
}

template <int BN, bool A_MN, bool B_MN, int STAGES, int EPI>
static void launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p, int device,
                             cudaStream_t stream) {
  using L = PairSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_pair_kernel<BN, A_MN, B_MN, STAGES, EPI>;
  static bool configured[64] = {false};
  if (!configured[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[device] = true;
  }
  p.num_m_tiles = (p.M + 255) / 256;
  p.num_n_tiles = (p.N + BN - 1) / BN;
  const int num_k = (p.K + kBK - 1) / kBK;
  if (p.splits < 1) p.splits = 1;
  p.k_blocks_per_split = (num_k + p.splits - 1) / p.splits;
  p.splits = (num_k + p.k_blocks_per_split - 1) / p.k_blocks_per_split;
  p.num_tiles = p.num_m_tiles * p.num_n_tiles * p.splits;
  if (p.splits > 1 && !p.accumulate)
    C10_CUDA_CHECK(cudaMemsetAsync(p.D, 0, (size_t)p.M * p.N * sizeof(float), stream));
  const int pairs = std::min(p.num_tiles, num_sms(device) / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
}

template <int BN>
static void dispatch_majors_pair(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                                 GemmParams& p, int device, cudaStream_t s) {
  constexpr int ST = 6;
  if (epi == kEpiGelu) return launch_gemm_pair<BN, false, false, ST, kEpiGelu>(ta, tb, p, device, s);
  if (epi == kEpiDGelu) return launch_gemm_pair<BN, false, true, ST, kEpiDGelu>(ta, tb, p, device, s);
  if (!a_mn && !b_mn) launch_gemm_pair<BN, false, false, ST, kEpiPlain>(ta, tb, p, device, s);
  else if (!a_mn && b_mn) launch_gemm_pair<BN, false, true, ST, kEpiPlain>(ta, tb, p, device, s);
  else if (a_mn && !b_mn) launch_gemm_pair<BN, true, false, ST, kEpiPlain>(ta, tb, p, device, s);
  else launch_gemm_pair<BN, true, true, ST, kEpiPlain>(ta, tb, p, device, s);
}

// 0: single-CTA tiles only; otherwise CTA pairs whenever M >= 256 (default). The environment
// variable MIA_GEMM_PAIR sets the initial value, `set_gemm_pair_mode` changes it at run time.
static std::atomic<int> g_pair_mode{[] {
  const char* v = std::getenv("MIA_GEMM_PAIR");
  return v == nullptr ? 2 : std::atoi(v);
}()};

static int pair_mode() { return g_pair_mode.load(std::memory_order_relaxed); }

int64_t set_gemm_pair_mode(int64_t mode) { return g_pair_mode.exchange((int)mode); }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Picks the N tile: 256 unless 128 gives noticeably better wave quantisation over the SMs.
static int choose_bn(int M, int N, int sms) {
  if (N <= 128) return 128;
  auto eff = [&](int bn) {
    const long tiles = (long)((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
    const long waves = (tiles + sms - 1) / sms;
    const double useful = (double)M * N;
    return useful / ((double)waves * sms * kBM * bn);
  };
  return eff(256) >= 0.85 * eff(128) ? 256 : 128;
}

// Same rule for 256 x BN tiles over CTA pairs. MIA_GEMM_BN=128|256 pins the choice (tuning runs).
static int choose_bn_pair(int M, int N, int sms) {
  static const int forced = [] {
    const char* v = std::getenv("MIA_GEMM_BN");
    return v == nullptr ? 0 : std::atoi(v);
  }();
  if (N <= 128) return 128;
  if (forced == 128 || forced == 256) return forced;
  const int pairs = sms / 2;
  auto eff = [&](int bn) {
    const long tiles = (long)((M + 255) / 256) * ((N + bn - 1) / bn);
    const long waves = (tiles + pairs - 1) / pairs;
    return (double)M * N / ((double)waves * pairs * 256 * bn);
  };
  return eff(256) >= 0.85 * eff(128) ? 256 : 128;
}

void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor d, c10::optional<torch::Tensor> bias,
          c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> gamma,
          c10::optional<torch::Tensor> aux_out, bool a_kmajor, bool b_kmajor, int64_t act, bool accumulate,
          c10::optional<torch::Tensor> colsum, double colsum_scale, c10::optional<torch::Tensor> a2,
          c10::optional<torch::Tensor> b2) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && d.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && d.dim() == 2, "gemm: 2-D tensors expected");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && d.is_contiguous(), "gemm: row-major operands expected");
  const int64_t M = a_kmajor ? a.size(0) : a.size(1);
  const int64_t K = a_kmajor ? a.size(1) : a.size(0);
  const int64_t N = b_kmajor ? b.size(0) : b.size(1);
  const int64_t Kb = b_kmajor ? b.size(1) : b.size(0);
  TORCH_CHECK(K == Kb, "gemm: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(d.size(0) == M && d.size(1) == N, "gemm: output shape mismatch");
  TORCH_CHECK(d.scalar_type() == at::kBFloat16 || d.scalar_type() == at::kFloat, "gemm: bf16 or fp32 output");
  // TMA needs 16-byte aligned rows: the contiguous extent of each operand (K for K-major, M or N
  // for MN-major) and the output's N must be multiples of 8 elements; the other extents are free
  // (out-of-range rows are zero-filled on load and skipped on store).
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  TORCH_CHECK(a_kmajor ? K % 8 == 0 : M % 8 == 0, "gemm: A's contiguous extent must be a multiple of 8");
  TORCH_CHECK(!b_kmajor || K % 8 == 0, "gemm: B's contiguous extent must be a multiple of 8");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm: leading dimensions must be multiples of 8");
  TORCH_CHECK(aligned16(a.data_ptr()) && aligned16(b.data_ptr()) && aligned16(d.data_ptr()),
              "gemm: 16-byte aligned base addresses expected");
  c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.D = d.data_ptr();
  p.d_fp32 = d.scalar_type() == at::kFloat;
  p.act = (int)act;
  p.accumulate = accumulate ? 1 : 0;
  p.err = error_word(device);
  auto check_vec = [&](const c10::optional<torch::Tensor>& t, const char* name) -> const float* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == N, "gemm: ",
                name, " must be a contiguous fp32 vector of length N");
    return t->data_ptr<float>();
  };
  auto check_mat = [&](const c10::optional<torch::Tensor>& t, const char* name) -> __nv_bfloat16* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->size(0) == M &&
                    t->size(1) == N && aligned16(t->data_ptr()),
                "gemm: ", name, " must be a contiguous, aligned bf16 (M, N) matrix");
    return reinterpret_cast<__nv_bfloat16*>(t->data_ptr());
  };
  p.bias = check_vec(bias, "bias");
  p.gamma = check_vec(gamma, "gamma");
  p.residual = check_mat(residual, "residual");
  p.aux = check_mat(aux, "aux");
  p.aux_out = check_mat(aux_out, "aux_out");
  TORCH_CHECK(act != kActDGelu || p.aux != nullptr, "gemm: GELU' needs aux");
  if (colsum.has_value()) {
    TORCH_CHECK(colsum->is_cuda() && colsum->scalar_type() == at::kFloat && colsum->is_contiguous() &&
                    colsum->numel() == N,
                "gemm: colsum must be a contiguous fp32 vector of length N");
    p.colsum = colsum->data_ptr<float>();
    p.colsum_scale = (float)colsum_scale;
  }

  // The CTA-pair kernels carry the activation epilogues only in the layouts the MLP uses: GELU with
  // both operands K-major (fc1 forward), GELU' with B N-major (dX of fc1). Other activated calls
  // take the single-CTA kernel, whose epilogue has everything.
  int epi = kEpiPlain;
  bool pair_ok = true;
  if (act == kActGelu) {
    epi = kEpiGelu;
    pair_ok = a_kmajor && b_kmajor;
  } else if (act == kActDGelu) {
    epi = kEpiDGelu;
    pair_ok = a_kmajor && !b_kmajor;
  }
  if (epi != kEpiPlain &&
      (d.scalar_type() == at::kFloat || gamma.has_value() || residual.has_value() || accumulate))
    pair_ok = false;
  if (a2.has_value() != b2.has_value()) TORCH_CHECK(false, "gemm: a2 and b2 come together");
  if (a2.has_value()) {
    TORCH_CHECK(a_kmajor && b_kmajor, "gemm: the second operand pair needs K-major A and B");
    TORCH_CHECK(a2->scalar_type() == at::kBFloat16 && b2->scalar_type() == at::kBFloat16 && a2->dim() == 2 &&
                    b2->dim() == 2 && a2->stride(1) == 1 && b2->stride(1) == 1 && a2->size(0) == M &&
                    b2->size(0) == N && a2->size(1) == b2->size(1) && a2->size(1) % 8 == 0 &&
                    a2->stride(0) % 8 == 0 && b2->stride(0) % 8 == 0 && aligned16(a2->data_ptr()) &&
                    aligned16(b2->data_ptr()),
                "gemm: a2 (M, K2) and b2 (N, K2) must be row-major bf16 with K2 % 8 == 0");
    p.K2 = (int)a2->size(1);
  }
  if (p.colsum != nullptr || p.K2 > 0) pair_ok = false;  // column sums and K2 live in the single-CTA kernel
  const bool use_pair = pair_mode() != 0 && M >= 256 && pair_ok;
  int bn = use_pair ? choose_bn_pair((int)M, (int)N, num_sms(device)) : choose_bn((int)M, (int)N, num_sms(device));
  static const bool bn_pinned = std::getenv("MIA_GEMM_BN") != nullptr;
  if (use_pair && !bn_pinned && N > 128) {
    // Measured per shape on the ViT-L MAE training step: activation epilogues are the slow part of
    // their GEMMs, so more, narrower tiles win; split-K weight gradients (fp32 out) prefer the wider
    // tile; plain GEMMs with a short K are epilogue-heavy too.
    const bool plain_f32_out = d.scalar_type() == at::kFloat && !bias.has_value() && !gamma.has_value() &&
                               !residual.has_value() && act == kActNone;
    if (act != kActNone) bn = 128;
    else if (plain_f32_out) bn = 256;
    else if (K <= 512) bn = 128;
  }
  // Split K when the output alone cannot fill the SMs and nothing in the epilogue needs the full
  // sum (the weight-gradient GEMMs: tokens are K, the output is a small fp32 matrix).
  p.splits = 1;
  const bool plain_fp32 = p.d_fp32 && !p.bias && !p.gamma && !p.residual && !p.aux && !p.aux_out && act == kActNone;
  if (plain_fp32 && p.colsum == nullptr && p.K2 == 0) {
    const long tiles = use_pair ? (long)((M + 255) / 256) * ((N + bn - 1) / bn)
                                : (long)((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
    const int sms = use_pair ? num_sms(device) / 2 : num_sms(device);
    const int k_blocks = (int)((K + kBK - 1) / kBK);
    if (2 * tiles <= sms) p.splits = (int)std::max(1L, std::min<long>(k_blocks / 4, sms / tiles));
  }
  // A tile: 128 rows x 64 K (K-major) or 64 M x 64 K per box, twice (M-major). B: BN rows (BN / 2
  // per CTA of a pair) x 64 K, or 64 N x 64 K boxes.
  const int b_rows = use_pair ? bn / 2 : bn;
  CUtensorMap ta = a_kmajor ? make_map(a.data_ptr(), K, M, a.stride(0), 64, kBM)
                            : make_map(a.data_ptr(), M, K, a.stride(0), 64, 64);
  CUtensorMap tb = b_kmajor ? make_map(b.data_ptr(), K, N, b.stride(0), 64, b_rows)
                            : make_map(b.data_ptr(), N, K, b.stride(0), 64, 64);
  CUtensorMap ta2 = ta, tb2 = tb;  // unused unless a second operand pair is given
  if (p.K2 > 0) {
    ta2 = make_map(a2->data_ptr(), p.K2, M, a2->stride(0), 64, kBM);
    tb2 = make_map(b2->data_ptr(), p.K2, N, b2->stride(0), 64, b_rows);
  }
  if (use_pair) {
    if (bn == 256) dispatch_majors_pair<256>(!a_kmajor, !b_kmajor, epi, ta, tb, p, device, stream);
    else dispatch_majors_pair<128>(!a_kmajor, !b_kmajor, epi, ta, tb, p, device, stream);
  } else if (bn == 256) {
    dispatch_majors<256>(!a_kmajor, !b_kmajor, ta, tb, ta2, tb2, p, device, stream);
  } else {
    dispatch_majors<128>(!a_kmajor, !b_kmajor, ta, tb, ta2, tb2, p, device, stream);
  }
}

// -------------------------------------------------------------- column sums (bias gradients)
// out[n] (+)= sum_m x[m, n]; x bf16 (M, N) row-major, N % 8 == 0. A CTA owns 256 columns (8 per
// lane) and a slab of rows split across its 8 warps; the warps are combined in shared memory and
// the CTA adds one partial per column. Each thread keeps 8 row loads in flight and the slab height
// gives about 4 CTAs per SM (the input is usually still in L2, so the kernel is latency- rather
// than bandwidth-bound); each column sees a few hundred atomics at most.
__global__ void __launch_bounds__(256) column_sum_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ out,
                                                         int M, int N, int rows_per_cta) {
  __shared__ float part[8][256];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int n = blockIdx.x * 256 + lane * 8;
  const int m_begin = blockIdx.y * rows_per_cta;
  const int m_end = min(M, m_begin + rows_per_cta);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (n < N) {
    int m = m_begin + warp;
    for (; m + 56 < m_end; m += 64) {
      uint4 u[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) u[r] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(m + 8 * r) * N + n));
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint32_t w[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          acc[2 * h] += bf16_lo(w[h]);
          acc[2 * h + 1] += bf16_hi(w[h]);
        }
      }
    }
    for (; m < m_end; m += 8) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * N + n));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        acc[2 * h] += bf16_lo(w[h]);
        acc[2 * h + 1] += bf16_hi(w[h]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[warp][lane * 8 + j] = acc[j];
  __syncthreads();
  const int c = threadIdx.x;  // one column of this CTA's 256
  if (blockIdx.x * 256 + c < N) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += part[w][c];
    atomicAdd(out + blockIdx.x * 256 + c, s);
  }
}

void column_sum(torch::Tensor x, torch::Tensor out, bool accumulate) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
              "column_sum: contiguous bf16 (M, N) expected");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == x.size(1),
              "column_sum: fp32 (N,) output expected");
  TORCH_CHECK(x.size(1) % 8 == 0, "column_sum: N must be a multiple of 8");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (!accumulate) C10_CUDA_CHECK(cudaMemsetAsync(out.data_ptr(), 0, out.numel() * 4, stream));
  const int M = (int)x.size(0), N = (int)x.size(1);
  if (M == 0) return;
  const int gx = (N + 255) / 256;
  const int gy = std::max(1, std::min((M + 63) / 64, (4 * num_sms(x.get_device()) + gx - 1) / gx));
  const int rows = (M + gy - 1) / gy;
  column_sum_kernel<<<dim3(gx, gy), 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                                      out.data_ptr<float>(), M, N, rows);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia
