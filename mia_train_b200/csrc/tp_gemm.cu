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
// Both are persistent tcgen05 GEMMs (one CTA per SM; warp 0 issues TMA, warp 1 issues tcgen05.mma
// into double-buffered TMEM accumulators, eight epilogue warps drain TMEM) over a static
// round-robin schedule of 128-row output tiles in a fixed block order, so every GEMM CTA gets the
// same number of tiles (+-1).
//
// Transfers are pushes. Between two B200s whose GEMMs keep both memories busy, TMA bulk pulls from
// the peer were measured at 210-330 GB/s while TMA stores into the peer kept ~620 GB/s per
// direction, so every byte crosses NVLink as a store into the receiver's memory, and the receiver's
// tensor cores then read it locally.
//
// all-gather -> GEMM. A few copy CTAs push this rank's rows, whole contiguous 128-row blocks in
// 32 KB bulk copies, into this rank's slot of every peer's gather area, and publish each block to
// every peer with a system-scope flag once its stores have landed. The GEMM CTAs compute this rank's
// blocks first, reading A straight from the caller's rows, then the peers' blocks in the order the
// peers push them, reading A from the local gather area once the block's flag is set. A store warp
// writes the A slices of every block's first N tile from shared memory into the gathered output,
// which the backward pass needs for dW.
//
// GEMM -> reduce-scatter. The peers' row blocks come first (block j of every peer in turn), this
// rank's own last. A peer tile is rounded to bf16 into one of two shared-memory staging
// tiles and sent by a store warp with TMA stores into the owner's receive slot; once its rows have
// landed it is counted against its block, and the CTA that completes a block publishes it to the
// owner. An own tile continues its K loop over the peers' partial tiles (TMA-loaded from this rank's
// receive slots once their flags are set) times columns of a 128 x 128 identity, and over the
// residual the same way when there is no LayerScale and no pre-activation output: the tensor core
// adds them exactly into the TMEM accumulator, so this rank's partial never leaves TMEM and the
// epilogue only applies bias, LayerScale and the residual before one bf16 store.
//
// Buffers and ordering. Gather and receive areas are double-buffered by the parity of a per-kind
// epoch counter kept on the device (advanced by the last CTA of every launch, so a captured CUDA
// graph replays correctly). A rank writes a peer's buffer e % 2 in launch e; that peer last read it
// in launch e - 2, and the writer has proof that the peer finished launch e - 2: in launch e - 1 it
// waited for data that the peer sent in its launch e - 1, which started only after the peer's launch
// e - 2 ended. Peer flags hold the epoch of the launch that published, so they only grow; local tile
// counters carry the epoch in their upper 32 bits. Every rank must issue the same sequence of these
// launches (every TP layer's forward and backward does). The all-gather and reduce-scatter areas are
// separate, since the two kinds interleave.
//
// Co-residency. CTAs wait on flags that CTAs of other GPUs publish, which in turn may wait on this
// GPU: the kernels are launched cooperatively, so all CTAs of a launch are resident together, and no
// CTA ever holds back data that a peer waits for while it waits itself. Every wait is bounded
// (%globaltimer); on expiry the kernel records an error code in the device error word and unwinds
// (drains its copies and MMAs, frees tensor memory) instead of hanging. No load uses cluster
// multicast: peers are only written, by plain TMA tile stores and bulk stores.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>
#include <vector>

#include "common.cuh"
#include "errors.h"
#include "gemm_common.cuh"

namespace mia {
namespace tp {

constexpr int kMaxWorld = 8;
constexpr int kMaxMBlocks = 2048;  // 128-row blocks of the gathered M: M <= 262144
constexpr int kEpi = 8;            // epilogue warps
constexpr int kAgThreads = 64 + 32 * kEpi + 32;  // producer, MMA, epilogue warps, store warp
constexpr int kRsThreads = 64 + 32 * kEpi + 32;  // producer, MMA, epilogue warps, store warp
constexpr int kRsBN = 128;
constexpr int kCopyChunk = 32768;  // bytes per bulk copy of an all-gather copy CTA
constexpr int kCopyCtaSlots = 6;   // chunks in flight per copy CTA

// Flag area of one rank (int32 units):
//   ag_ready[src][block]  written by src: its rows of gathered block `block` are in our gather area
//   rs_ready[src][block]  written by src: its partial rows of block `block` are in our receive slot
//   ctl[16]               local: epochs and exit counters
//   tiles[block]          local int64: (epoch << 32) | N tiles of block `block` sent (reduce-scatter)
constexpr int kAgReady = 0;
constexpr int kRsReady = kAgReady + kMaxWorld * kMaxMBlocks;
constexpr int kCtl = kRsReady + kMaxWorld * kMaxMBlocks;
constexpr int kCtlAgEpoch = 0, kCtlAgExit = 1, kCtlRsEpoch = 2, kCtlRsExit = 3;
constexpr int kTiles = kCtl + 16;
constexpr int kFlagInts = kTiles + 2 * kMaxMBlocks;
static_assert(kTiles % 2 == 0, "64-bit flag words must be 8-byte aligned");

// Optional per-CTA timeline (globaltimer ns) of the last launch of each kernel, for tuning: enabled
// with MIA_TP_TRACE=1, read with tp_trace_read(). kTracePoints events per CTA.
constexpr int kTraceCtas = 160;
constexpr int kTracePoints = 8;

struct Peers {
  int64_t p[kMaxWorld];
};

__device__ __forceinline__ int64_t pick(const Peers& p, int i) {
  int64_t r = p.p[0];
#pragma unroll
  for (int j = 1; j < kMaxWorld; ++j) r = (i == j) ? p.p[j] : r;
  return r;
}

__device__ __forceinline__ void trace_mark(long long* trace, int point) {
  if (trace != nullptr) trace[blockIdx.x * kTracePoints + point] = (long long)globaltimer_ns();
}

__device__ __forceinline__ void st_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Bounded wait until *flag >= target (system scope). False on timeout (error recorded) or when
// another role of this CTA has aborted.
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

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
// 1-D bulk copies (no tensor map): global -> shared with an mbarrier, shared -> global in a group.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store_1d(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all_but_one() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all_but_three() { asm volatile("cp.async.bulk.wait_group 3;" ::: "memory"); }

struct TpShape {
  int M, N, K;      // gathered rows, output columns, reduction length
  int S;            // rows per rank (M = S * world)
  int rank, world;
  int num_blocks;   // ceil(M / 128)
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ------------------------------------------------------------------------------- all-gather GEMM
struct AgParams {
  GemmParams g;                  // M = gathered rows; D, bias, aux, aux_out, act, err
  TpShape s;
  Peers flags;
  Peers gather;                  // every rank's gather area: [parity][src][S][K] bf16
  int64_t gather_parity_bytes;
  const __nv_bfloat16* a_local;  // this rank's rows (S, K)
  int copy_ctas;                 // CTAs [0, copy_ctas) push this rank's rows; the rest run the GEMM
  uint64_t timeout_ns;
  long long* trace;  // points: 0 start, 1 first-N-tile slices stored, 2 first block pushed, 3 all blocks
                     // pushed, 4 producer reached the peers' tiles, 5 MMA done, 6 epilogue done, 7 exit
};

// Tensor maps: the gathered output, this rank's rows, and this rank's gather area as a 4-D
// (K, S, src, parity) array.
struct AgMaps {
  CUtensorMap full;    // (K, M) gathered A, local
  CUtensorMap local;   // (K, S) this rank's rows, local
  CUtensorMap gather;  // (K, S, W, 2) the peers' rows pushed here
};

template <int BN, int STAGES>
struct AgSmem {
  static constexpr int kBTileBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kGemmBar = STAGES * kStageBytes;
  static constexpr int kCopyBar = kCopyCtaSlots * kCopyChunk;
  static constexpr int kBarOffset = kGemmBar > kCopyBar ? kGemmBar : kCopyBar;
  static constexpr int kBytes = kBarOffset + 1024 + 512;
};

// Ordered block index -> gathered row block: this rank's blocks first, then the peers' blocks
// interleaved by distance (block j of the next rank, of the rank after, ..., then block j + 1), the
// order in which every rank's copy CTAs push them.
__device__ __forceinline__ int ag_block(const TpShape& s, int nloc, int bi) {
  if (bi < nloc) return s.rank * nloc + bi;
  const int ri = bi - nloc, d = ri % (s.world - 1) + 1, j = ri / (s.world - 1);
  return ((s.rank + d) % s.world) * nloc + j;
}

// Copy CTA c of C: pushes this rank's row blocks c, c + C, ... to every peer. A block (128
// contiguous rows) is read in 32 KB bulk loads (six in flight) and each chunk is written by bulk
// stores into the same place of every peer's gather area (this rank's slot); after a block's last
// chunk the thread waits for the block's stores to land and publishes it to every peer with a
// system-scope flag. The stores never hold a slot (only their shared-memory reads do). One thread
// works; nothing here waits on another GPU.
__device__ __forceinline__ void ag_copy_cta(const AgParams& P, uint8_t* smem, int nloc, int epoch, int par,
                                            volatile int* abort_flag) {
  const TpShape& s = P.s;
  const int C = P.copy_ctas, c = blockIdx.x;
  uint64_t* cbar = reinterpret_cast<uint64_t*>(smem + kCopyCtaSlots * kCopyChunk);
  const int64_t block_bytes = 128LL * s.K * 2;
  const int chunks = (int)((block_bytes + kCopyChunk - 1) / kCopyChunk);
  const int n_items = nloc > c ? (nloc - 1 - c) / C + 1 : 0;
  const int total = n_items * chunks;
  auto item_local = [&](int it) { return c + it * C; };  // this rank's block index
  auto chunk_bytes = [&](int ch) {
    const int64_t rest = block_bytes - (int64_t)ch * kCopyChunk;
    return (uint32_t)(rest < kCopyChunk ? rest : kCopyChunk);
  };
  int issued = 0, consumed = 0, published = 0;
  bool ok = true;
  auto publish_upto = [&](int items) {
    if (published >= items) return;
    fence_proxy_async_global();
    fence_acq_rel_sys();
    for (; published < items; ++published) {
      const int mb = s.rank * nloc + item_local(published);
      for (int r = 0; r < s.world; ++r)
        if (r != s.rank)
          st_release_sys(reinterpret_cast<int*>(pick(P.flags, r)) + kAgReady + s.rank * kMaxMBlocks + mb, epoch);
      if (published == 0) trace_mark(P.trace, 2);
    }
  };
  auto issue = [&](int g) {
    const int it = g / chunks, ch = g - it * chunks;
    const int slot = g % kCopyCtaSlots;
    const uint8_t* from = reinterpret_cast<const uint8_t*>(P.a_local) + (int64_t)item_local(it) * block_bytes +
                          (int64_t)ch * kCopyChunk;
    mbar_arrive_expect_tx(&cbar[slot], chunk_bytes(ch));
    bulk_load_1d(smem + slot * kCopyChunk, from, chunk_bytes(ch), &cbar[slot]);
  };
  for (; issued < total && issued < kCopyCtaSlots; ++issued) issue(issued);
  const int64_t slot_off = (int64_t)par * P.gather_parity_bytes + (int64_t)s.rank * s.S * s.K * 2;
  for (int g = 0; g < total; ++g) {
    const int slot = g % kCopyCtaSlots;
    if (!mbar_wait(&cbar[slot], (g / kCopyCtaSlots) & 1, abort_flag, P.g.err, kErrTpChunkWait)) {
      ok = false;
      break;
    }
    consumed = g + 1;
    const int it = g / chunks, ch = g - it * chunks;
    const int64_t off = slot_off + (int64_t)item_local(it) * block_bytes + (int64_t)ch * kCopyChunk;
    for (int r = 0; r < s.world; ++r)
      if (r != s.rank)
        bulk_store_1d(reinterpret_cast<uint8_t*>(pick(P.gather, r)) + off, smem + slot * kCopyChunk, chunk_bytes(ch));
    bulk_commit();
    bulk_wait_read();  // the slot may be refilled
    if (issued < total) issue(issued++);
    if (ch == chunks - 1) {
      // the block's last chunk: wait for its stores (the next loads stay in flight) and publish it
      // at once, so that the peers' GEMMs can start on it
      bulk_wait_all();
      publish_upto(it + 1);
    }
  }
  bulk_wait_all();
  if (ok) {
    publish_upto(n_items);
  } else {
    for (int g = consumed; g < issued; ++g)  // loads still in flight write shared memory
      mbar_wait(&cbar[g % kCopyCtaSlots], (g / kCopyCtaSlots) & 1, nullptr, nullptr, 0);
  }
  trace_mark(P.trace, 3);
}

// GEMM CTA warp roles: 0 TMA producer, 1 MMA issuer, 2..9 epilogue, 10 store warp.
//
// Tiles (128 rows x BN) are dealt round-robin over the GEMM CTAs in block order, this rank's blocks
// first. A peer's block is read from the gather area once its flag is set. The store warp writes
// the A slices of each block's first N tile, straight from the stage, into the gathered output
// before the stage is reused.
template <int BN, bool B_MN, int STAGES, int EPI>
__global__ void __launch_bounds__(kAgThreads, 1)
    tp_ag_gemm_kernel(const __grid_constant__ AgMaps maps, const __grid_constant__ CUtensorMap tmB, const AgParams P) {
  using L = AgSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const GemmParams& p = P.g;
  const TpShape& s = P.s;
  const int nloc = s.world > 1 ? s.S / 128 : s.num_blocks;
  int* my_flags = reinterpret_cast<int*>(pick(P.flags, s.rank));
  const int epoch = *reinterpret_cast<const volatile int*>(my_flags + kCtl + kCtlAgEpoch) + 1;
  const int par = epoch & 1;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kBarOffset + 512);

  if ((int)blockIdx.x < P.copy_ctas) {
    // ================= copy CTA
    uint64_t* cbar = reinterpret_cast<uint64_t*>(smem + kCopyCtaSlots * kCopyChunk);
    if (threadIdx.x == 0) {
      for (int i = 0; i < kCopyCtaSlots; ++i) mbar_init(&cbar[i], 1);
      *abort_flag = 0;
      fence_barrier_init();
      trace_mark(P.trace, 0);
    }
    __syncthreads();
    if (threadIdx.x == 0) ag_copy_cta(P, smem, nloc, epoch, par, abort_flag);
    __syncthreads();
  } else {
    // ================= GEMM CTA
    const int cta = blockIdx.x - P.copy_ctas, G = gridDim.x - P.copy_ctas;
    uint8_t* smA = smem;
    uint8_t* smB = smem + STAGES * kATileBytes;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* tfull_bar = empty_bar + STAGES;
    uint64_t* tempty_bar = tfull_bar + 2;
    uint64_t* drain_bar = tempty_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    constexpr uint32_t kTmemCols = 2 * BN;
    const int num_k = (p.K + kBK - 1) / kBK;
    const int num_n = (p.N + BN - 1) / BN;
    const int num_tiles = s.num_blocks * num_n;

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
      fence_barrier_init();
      prefetch_tensormap(&maps.full);
      prefetch_tensormap(&maps.local);
      prefetch_tensormap(&tmB);
      trace_mark(P.trace, 0);
    }
    if (warp == 1) {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    constexpr int kStoreWarp = 2 + kEpi;

    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0;
        bool ok = true, marked = false;
        constexpr uint32_t kTx = kATileBytes + L::kBTileBytes;
        for (int t = cta; t < num_tiles && ok; t += G) {
          const int bi = t / num_n, nt = t - bi * num_n;
          const int mb = ag_block(s, nloc, bi);
          const bool local = bi < nloc;
          const int m0 = mb * 128, n0 = nt * BN;
          const int src = mb / nloc;
          if (!local) {
            if (!marked) {
              trace_mark(P.trace, 4);
              marked = true;
            }
            // the owner must have pushed the block into our gather area before the first load
            if (!wait_flag(my_flags + kAgReady + src * kMaxMBlocks + mb, epoch, P.timeout_ns, abort_flag, p.err,
                           kErrTpChunkWait)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
          }
          for (int kb = 0; kb < num_k; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrGemmProducerWait)) {
              ok = false;
              break;
            }
            const int k0 = kb * kBK;
            mbar_arrive_expect_tx(&full_bar[stage], kTx);
            uint8_t* a_dst = smA + stage * kATileBytes;
            uint8_t* b_dst = smB + stage * L::kBTileBytes;
            if (local) tma_load_2d(a_dst, &maps.local, &full_bar[stage], k0, m0 - s.rank * s.S);
            else tma_load_4d(a_dst, &maps.gather, &full_bar[stage], k0, m0 - src * s.S, src, par);
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
        for (int t = cta; t < num_tiles && ok; t += G) {
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
        if (!ok && any) {
          tc_commit(drain_bar);
          mbar_wait(drain_bar, 0, nullptr, nullptr, 0);
        }
        trace_mark(P.trace, 5);
      }
    } else if (warp == kStoreWarp) {
      if (lane == 0) {
        // ---------------- store warp: first-N-tile A slices -> gathered output
        // Every block's A slices pass through this CTA's stages for its first N tile (this rank's
        // rows from the caller's matrix, a peer's from the gather area): the warp writes each one
        // into the gathered output; the stage is released once the store has read it.
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = cta; t < num_tiles && ok; t += G) {
          const int bi = t / num_n, nt = t - bi * num_n;
          const int mb = ag_block(s, nloc, bi);
          for (int kb = 0; kb < num_k; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrTpChunkWait)) {
              ok = false;
              break;
            }
            if (nt == 0) {
              tma_store_2d(&maps.full, smA + stage * kATileBytes, kb * kBK, mb * 128);
              bulk_commit();
              bulk_wait_read();
            }
            mbar_arrive(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        bulk_wait_all();
        trace_mark(P.trace, 1);
      }
    } else if (warp >= 2 && warp < 2 + kEpi) {
      // ---------------- epilogue warps 2..9
      const int lane_group = warp % 4;
      const int col_part = (warp - 2) / 4;  // two column halves
      constexpr int kPartCols = BN / 2;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = cta; t < num_tiles; t += G) {
        const int bi = t / num_n, nt = t - bi * num_n;
        const int m = ag_block(s, nloc, bi) * 128 + lane_group * 32 + lane;
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrGemmEpilogueWait)) break;
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
      if (warp == 2 && lane == 0) trace_mark(P.trace, 6);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, kTmemCols);
    }
  }
  if (threadIdx.x == 0) {
    trace_mark(P.trace, 7);
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
  Peers flags;
  // epilogue of this rank's rows: out = residual + gamma * (sum + bias); `pre_out` keeps sum + bias
  __nv_bfloat16* out;
  const float* bias;
  const float* gamma;
  const __nv_bfloat16* residual;
  __nv_bfloat16* pre_out;
  int fold_residual;  // the residual enters the accumulator through the identity MMA
  uint64_t timeout_ns;
  long long* trace;  // points: 0 start, 1 MMA done, 2 epilogue done, 3 peer tiles landed,
                     // 4 first own block's partials present, 7 exit
};

// Every owner's receive area as a 4-D (N, S, src slot, parity) bf16 array, written by TMA stores
// (and read back, for this rank's own rows, as A tiles of the identity MMA); a 128 x 128 identity in
// the B operand's layout; this rank's residual rows (N, S) when they are folded in the same way.
struct RsMaps {
  CUtensorMap recv[kMaxWorld];
  CUtensorMap ident;
  CUtensorMap res;
};

template <int STAGES>
struct RsSmem {
  static constexpr int kBTileBytes = kRsBN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  // two bf16 output tiles, each kRsBN / 64 slabs of 128 rows x 128 bytes in the TMA 128-byte swizzle
  static constexpr int kStagingBytes = 128 * kRsBN * 2;
  static constexpr int kStagingOffset = STAGES * kStageBytes;
  static constexpr int kBarOffset = kStagingOffset + 2 * kStagingBytes;
  static constexpr int kBytes = kBarOffset + 1024 + 512;
};

// Ordered block index -> row block. Step j sends block j of every peer (interleaved, so every
// peer's link is busy) and then computes this rank's own block j - delta: own blocks trail by
// `delta` steps, so that by the time one is computed the peers (which follow the same order) have
// sent their partials of it. With delta = nloc every own block comes last.
__device__ __forceinline__ int rs_block(const TpShape& s, int nloc, int delta, int bi) {
  if (s.world == 1) return bi;
  const int W = s.world, a = delta * (W - 1);
  if (bi < a) return ((s.rank + bi % (W - 1) + 1) % W) * nloc + bi / (W - 1);
  const int r = bi - a;
  if (r < (nloc - delta) * W) {
    const int j = delta + r / W, k = r % W;
    return k < W - 1 ? ((s.rank + k + 1) % W) * nloc + j : s.rank * nloc + j - delta;
  }
  return s.rank * nloc + nloc - delta + (r - (nloc - delta) * W);
}

// Counts one finished tile of `word`'s block in this launch; true for the block's last tile.
__device__ __forceinline__ bool count_tile(unsigned long long* word, unsigned long long ep_hi, int tiles_per_block) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(word);
  while (true) {
    const unsigned long long want = ((cur & 0xFFFFFFFF00000000ull) == ep_hi) ? cur + 1 : (ep_hi | 1ull);
    const unsigned long long prev = atomicCAS(word, cur, want);
    if (prev == cur) return (int)(want & 0xFFFFFFFFull) == tiles_per_block;
    cur = prev;
  }
}

__device__ __forceinline__ void add_bf16x32(float (&v)[32], const uint4 (&u)[4]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t w[4] = {u[c].x, u[c].y, u[c].z, u[c].w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      v[8 * c + 2 * h] += bf16_lo(w[h]);
      v[8 * c + 2 * h + 1] += bf16_hi(w[h]);
    }
  }
}

// One 32-column chunk of one row of this rank's output. The accumulator already holds this rank's
// partial plus the peers' (and the residual, when folded); what is left is bias, `pre_out`,
// LayerScale and the residual add. `res` is the chunk's residual, loaded before the TMEM load.
__device__ __forceinline__ void rs_own_chunk(const RsParams& P, int row, int n, const uint32_t (&r)[32],
                                             const uint4 (&res)[4]) {
  const TpShape& s = P.s;
  if (row >= s.S || n >= s.N) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  const int64_t off = (int64_t)row * s.N + n;
  const bool add_res = P.residual != nullptr && !P.fold_residual;
  if (n + 32 <= s.N) {
    if (P.bias != nullptr) {
      const float4* b4 = reinterpret_cast<const float4*>(P.bias + n);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 bb = __ldg(b4 + c);
        v[4 * c] += bb.x; v[4 * c + 1] += bb.y; v[4 * c + 2] += bb.z; v[4 * c + 3] += bb.w;
      }
    }
    if (P.pre_out != nullptr) {
      uint4* dst = reinterpret_cast<uint4*>(P.pre_out + off);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        dst[c] = make_uint4(pack_bf16x2(v[8 * c + 0], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                            pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
    }
    if (P.gamma != nullptr) {
      const float4* g4 = reinterpret_cast<const float4*>(P.gamma + n);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 gg = __ldg(g4 + c);
        v[4 * c] *= gg.x; v[4 * c + 1] *= gg.y; v[4 * c + 2] *= gg.z; v[4 * c + 3] *= gg.w;
      }
    }
    if (add_res) add_bf16x32(v, res);
    uint4* dst = reinterpret_cast<uint4*>(P.out + off);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      dst[c] = make_uint4(pack_bf16x2(v[8 * c + 0], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                          pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (n + j >= s.N) continue;
      float x = v[j];
      if (P.bias != nullptr) x += P.bias[n + j];
      if (P.pre_out != nullptr) P.pre_out[off + j] = __float2bfloat16_rn(x);
      if (P.gamma != nullptr) x *= P.gamma[n + j];
      if (add_res) x += __bfloat162float(P.residual[off + j]);
      P.out[off + j] = __float2bfloat16_rn(x);
    }
  }
}

// Warp roles: 0 TMA producer, 1 MMA issuer, 2..9 epilogue, 10 store warp.
template <bool B_MN, int STAGES>
__global__ void __launch_bounds__(kRsThreads, 1)
    tp_gemm_rs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ RsMaps maps, const RsParams P) {
  using L = RsSmem<STAGES>;
  constexpr int BN = kRsBN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kATileBytes;
  uint8_t* staging = smem + L::kStagingOffset;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* sfull_bar = drain_bar + 1;   // [2] staging tile written (epilogue threads)
  uint64_t* sempty_bar = sfull_bar + 2;  // [2] staging tile read by the TMA stores (store warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const TpShape& s = P.s;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr uint32_t kTmemCols = 2 * BN;
  const int num_k = (s.K + kBK - 1) / kBK;
  const int num_n = (s.N + BN - 1) / BN;
  const int nloc = s.world > 1 ? s.S / 128 : s.num_blocks;
  const int num_tiles = s.num_blocks * num_n;
  // Own blocks come after every peer block. (Trailing the peers' by three rounds of tiles instead, so
  // that their identity MMAs overlap the sends, measured 4-17% slower at two ranks: each own tile
  // must first flush the store warp's pending tile counts.)
  const int delta = s.world > 1 ? nloc : 0;
  auto is_own = [&](int mb) { return s.world == 1 || mb / nloc == s.rank; };
  // own tiles continue their K loop over the peers' partials (and the residual) times the identity
  const int extra = 2 * (s.world - 1) + (P.fold_residual ? 2 : 0);
  int* my_flags = reinterpret_cast<int*>(pick(P.flags, s.rank));
  const int epoch = *reinterpret_cast<const volatile int*>(my_flags + kCtl + kCtlRsEpoch) + 1;
  const int par = epoch & 1;
  const unsigned long long ep_hi = (unsigned long long)(unsigned)epoch << 32;
  unsigned long long* tile_count = reinterpret_cast<unsigned long long*>(my_flags + kTiles);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * kEpi);
      mbar_init(&sfull_bar[a], 32 * kEpi);
      mbar_init(&sempty_bar[a], 1);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    trace_mark(P.trace, 0);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  constexpr int kStoreWarp = 2 + kEpi;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true, marked = false;
      constexpr uint32_t kTx = kATileBytes + L::kBTileBytes;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int bi = t / num_n, nt = t - bi * num_n;
        const int mb = rs_block(s, nloc, delta, bi);
        const int m0 = mb * 128, n0 = nt * BN;
        const int slices = num_k + (is_own(mb) ? extra : 0);
        for (int kb = 0; kb < slices; ++kb) {
          if (kb == num_k && s.world > 1) {
            // the peers' partial rows of this block must be in our receive slots before we read them
            bool ready = true;
            for (int q = 0; q < s.world && ready; ++q)
              if (q != s.rank)
                ready = wait_flag(my_flags + kRsReady + q * kMaxMBlocks + mb, epoch, P.timeout_ns, abort_flag, P.err,
                                  kErrTpSlotWait);
            if (!ready) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
            if (!marked) {
              trace_mark(P.trace, 4);
              marked = true;
            }
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, P.err, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kTx);
          uint8_t* a_dst = smA + stage * kATileBytes;
          uint8_t* b_dst = smB + stage * L::kBTileBytes;
          const CUtensorMap* bmap = &tmB;
          int bn0 = n0, bk0 = kb * kBK;
          if (kb < num_k) {
            tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * kBK, m0);
          } else {
            // identity MMA: A = a peer's partial tile (or the residual), B = 64 columns of I
            const int e = kb - num_k, half = e & 1, src = e >> 1;  // src-th peer, or the residual past them
            const int own_row = m0 - s.rank * s.S;
            if (src < s.world - 1)
              tma_load_4d(a_dst, &maps.recv[s.rank], &full_bar[stage], n0 + 64 * half, own_row,
                          (s.rank + 1 + src) % s.world, par);
            else
              tma_load_2d(a_dst, &maps.res, &full_bar[stage], n0 + 64 * half, own_row);
            bmap = &maps.ident;
            bn0 = 0;
            bk0 = 64 * half;
          }
          if (!B_MN) {
            tma_load_2d(b_dst, bmap, &full_bar[stage], bk0, bn0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, bmap, &full_bar[stage], bn0 + 64 * j, bk0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
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
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, P.err, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int slices = num_k + (is_own(rs_block(s, nloc, delta, t / num_n)) ? extra : 0);
        for (int kb = 0; kb < slices; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, P.err, kErrGemmMmaWait)) {
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
      if (!ok && any) {
        tc_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, nullptr, 0);
      }
      trace_mark(P.trace, 1);
    }
  } else if (warp >= 2 && warp < 2 + kEpi) {
    // ---------------- epilogue warps
    // Warp (lane quarter, column half) owns rows [32 q, 32 q + 32) x columns [64 h, 64 h + 64) of a
    // tile: for a peer's tile exactly one 128-byte-wide slab of the staging tile, each row's eight
    // 16-byte chunks XOR-permuted by row % 8 (the TMA 128-byte swizzle).
    const int lane_group = warp % 4;
    const int col_part = (warp - 2) / 4;
    const int row = lane_group * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    int jp = 0;  // peer tiles staged so far
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int bi = t / num_n, nt = t - bi * num_n;
      const int mb = rs_block(s, nloc, delta, bi);
      const bool own = is_own(mb);
      const int b = jp & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, P.err, kErrGemmEpilogueWait)) break;
      if (!own && !mbar_wait(&sempty_bar[b], ((jp >> 1) & 1) ^ 1, abort_flag, P.err, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(lane_group * 32) << 16) + acc * BN + col_part * 64;
      if (own) {
        const int own_row = mb * 128 - s.rank * s.S + row;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const int n = nt * BN + col_part * 64 + c * 32;
          uint4 res[4] = {};
          if (P.residual != nullptr && !P.fold_residual && own_row < s.S && n + 32 <= s.N) {
            const uint4* src = reinterpret_cast<const uint4*>(P.residual + (int64_t)own_row * s.N + n);
#pragma unroll
            for (int q = 0; q < 4; ++q) res[q] = __ldg(src + q);
          }
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait_regs(r);
          rs_own_chunk(P, own_row, n, r, res);
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
      } else {
        uint8_t* slab = staging + b * L::kStagingBytes + col_part * 16384 + row * 128;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait_regs(r);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = make_uint4(pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1])),
                                       pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                                       pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                                       pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
            *reinterpret_cast<uint4*>(slab + (((c * 4 + q) ^ (row & 7)) * 16)) = v;
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);  // the MMA may refill this accumulator
        fence_proxy_async_smem();       // the staging writes are read by the TMA engine next
        mbar_arrive(&sfull_bar[b]);
        ++jp;
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (warp == 2 && lane == 0) trace_mark(P.trace, 2);
  } else if (warp == kStoreWarp) {
    if (lane == 0 && s.world > 1) {
      // ---------------- store warp: staged peer tiles -> owner's receive slot
      // A staging tile is released once its stores have read it (one tile later, so the wait is
      // normally over); a tile is counted against its block once its rows have landed (three tiles
      // later, or at once when this CTA reaches one of its own tiles, whose producer may wait on the
      // peers). Only the CTA that completes a block pays for a system-scope release.
      int ring[4] = {-1, -1, -1, -1};  // blocks of the last four tiles issued
      int j = 0;
      bool ok = true;
      auto tile_landed = [&](int mb) {
        fence_proxy_async_global();
        fence_acq_rel_gpu();
        if (count_tile(tile_count + mb, ep_hi, num_n)) {
          fence_acq_rel_sys();
          st_release_sys(reinterpret_cast<int*>(pick(P.flags, mb / nloc)) + kRsReady + s.rank * kMaxMBlocks + mb,
                         epoch);
        }
      };
      int landed = 0;  // tiles counted so far
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int bi = t / num_n, nt = t - bi * num_n;
        const int mb = rs_block(s, nloc, delta, bi);
        if (is_own(mb)) {
          // this CTA's producer may now wait for the peers' partials, and the peers for ours: count
          // every tile sent so far before that can happen
          bulk_wait_all();
          for (; landed < j; ++landed) tile_landed(ring[landed & 3]);
          continue;
        }
        const int b = j & 1;
        if (!mbar_wait(&sfull_bar[b], (j >> 1) & 1, abort_flag, P.err, kErrGemmEpilogueWait)) {
          ok = false;
          break;
        }
        const int owner = mb / nloc;
        const uint8_t* tile = staging + b * L::kStagingBytes;
#pragma unroll
        for (int h = 0; h < BN / 64; ++h)
          if (nt * BN + h * 64 < s.N)
            tma_store_4d(&maps.recv[owner], tile + h * 16384, nt * BN + h * 64, mb * 128 - owner * s.S, s.rank, par);
        bulk_commit();
        ring[j & 3] = mb;
        bulk_wait_read_all_but_one();  // tile j - 1's staging buffer has been read
        if (j >= 1) mbar_arrive(&sempty_bar[(j - 1) & 1]);
        bulk_wait_all_but_three();  // tile j - 3's rows are in the owner's slot
        for (; landed <= j - 3; ++landed) tile_landed(ring[landed & 3]);
        ++j;
      }
      bulk_wait_all();
      if (ok)
        for (; landed < j; ++landed) tile_landed(ring[landed & 3]);
      trace_mark(P.trace, 3);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) {
    trace_mark(P.trace, 7);
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

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// bf16 tensor map of `rank` dimensions (innermost first) with a 64 x 128 box in the 128-byte swizzle.
static CUtensorMap area_map(int64_t base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                            const char* what) {
  CUtensorMap map;
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, reinterpret_cast<void*>(base), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (", what, ") failed with ", (int)r);
  return map;
}

// Trace buffers ([all-gather, reduce-scatter][kTraceCtas][kTracePoints] int64 per device), allocated
// on first use when MIA_TP_TRACE=1; nullptr otherwise.
static long long* trace_buffer(int device, int kind) {
  static const bool enabled = [] {
    const char* v = std::getenv("MIA_TP_TRACE");
    return v != nullptr && std::atoi(v) != 0;
  }();
  if (!enabled) return nullptr;
  static long long* buf[64] = {nullptr};
  if (buf[device] == nullptr) {
    const size_t bytes = 2 * kTraceCtas * kTracePoints * sizeof(long long);
    C10_CUDA_CHECK(cudaMalloc(&buf[device], bytes));
    C10_CUDA_CHECK(cudaMemset(buf[device], 0, bytes));
  }
  return buf[device] + (size_t)kind * kTraceCtas * kTracePoints;
}

template <int BN, bool B_MN, int EPI>
static void launch_ag(const AgMaps& maps, const CUtensorMap& tb, const AgParams& prm, int grid, cudaStream_t st,
                      int device) {
  constexpr int ST = BN == 256 ? 4 : 6;
  using L = AgSmem<BN, ST>;
  static_assert(L::kBytes <= 232448, "all-gather GEMM shared memory exceeds the per-CTA limit");
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

template <bool B_MN>
static void launch_rs(const CUtensorMap& ta, const CUtensorMap& tb, const RsMaps& maps, const RsParams& prm, int grid,
                      cudaStream_t st, int device) {
  constexpr int ST = 5;
  using L = RsSmem<ST>;
  static_assert(L::kBytes <= 232448, "reduce-scatter GEMM shared memory exceeds the per-CTA limit");
  auto kern = tp_gemm_rs_kernel<B_MN, ST>;
  static bool configured[64] = {false};
  if (!configured[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[device] = true;
  }
  coop_launch(kern, grid, kRsThreads, L::kBytes, st, ta, tb, maps, prm);
}

}  // namespace tp

// D = epi(gather(A) . B^T). a_local (S, K) bf16 this rank's rows; b (N, K) (b_kmajor) or (K, N);
// out (M, N) bf16; a_full (M, K) bf16 receives the gathered A. `gather_peers[q]` is rank q's gather
// area (two parities of `gather_parity_bytes`, each holding one (S, K) slot per source rank),
// `flag_peers[q]` its flag area.
void tp_ag_gemm(at::Tensor a_local, at::Tensor b, at::Tensor out, at::Tensor a_full, c10::optional<at::Tensor> bias,
                c10::optional<at::Tensor> aux, c10::optional<at::Tensor> aux_out, bool b_kmajor, int64_t act,
                std::vector<int64_t> flag_peers, std::vector<int64_t> gather_peers, int64_t gather_parity_bytes,
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
  TORCH_CHECK((int64_t)world * S * K * 2 <= gather_parity_bytes, "tp_ag_gemm: gather area too small (",
              gather_parity_bytes, " bytes for ", (int64_t)world * S * K * 2, ")");
  TORCH_CHECK(gather_parity_bytes % 256 == 0, "tp_ag_gemm: gather parity stride must be a multiple of 256 bytes");
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
  prm.gather = to_peers(gather_peers, world, "tp_ag_gemm gather");
  prm.gather_parity_bytes = gather_parity_bytes;
  prm.a_local = reinterpret_cast<const __nv_bfloat16*>(a_local.data_ptr());
  prm.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms * 1e6 : 5e9);
  prm.trace = trace_buffer(device, 0);

  const int bn = N <= 128 ? 128 : 256;
  const int64_t tiles = prm.s.num_blocks * ((N + bn - 1) / bn);
  // With peers, CTAs [0, copy_ctas) push this rank's rows: 16 for two ranks, 4 more per extra peer
  // (up to 32); MIA_TP_COPY_CTAS overrides.
  static const int copy_env = [] {
    const char* v = std::getenv("MIA_TP_COPY_CTAS");
    return v == nullptr ? -1 : std::atoi(v);
  }();
  const int sms = sm_count(device);
  const int copy_default = std::min(32, 16 + 4 * (world - 2));
  prm.copy_ctas = world == 1 ? 0 : std::max(1, std::min(copy_env >= 0 ? copy_env : copy_default, sms / 2));
  const int grid = (int)std::min<int64_t>(tiles + prm.copy_ctas, sms);
  const int epi = act == kActGelu ? kEpiGelu : (act == kActDGelu ? kEpiDGelu : kEpiPlain);
  AgMaps maps{};
  maps.full = make_bf16_map(a_full.data_ptr(), K, M, K, 64, kBM);
  maps.local = make_bf16_map(a_local.data_ptr(), K, S, K, 64, kBM);
  {
    const cuuint64_t dims[4] = {(cuuint64_t)K, (cuuint64_t)S, (cuuint64_t)world, 2};
    const cuuint64_t strides[3] = {(cuuint64_t)(K * 2), (cuuint64_t)(S * K * 2), (cuuint64_t)gather_parity_bytes};
    maps.gather = area_map(prm.gather.p[rank], 4, dims, strides, "gather area");
  }
  CUtensorMap tb = b_kmajor ? make_bf16_map(b.data_ptr(), K, N, K, 64, bn) : make_bf16_map(b.data_ptr(), N, K, N, 64, 64);
  if (bn == 256) {
    if (b_kmajor) dispatch_ag_epi<256, false>(epi, maps, tb, prm, grid, stream, device);
    else dispatch_ag_epi<256, true>(epi, maps, tb, prm, grid, stream, device);
  } else {
    if (b_kmajor) dispatch_ag_epi<128, false>(epi, maps, tb, prm, grid, stream, device);
    else dispatch_ag_epi<128, true>(epi, maps, tb, prm, grid, stream, device);
  }
}

// O_r = residual + gamma * (sum_q (A_q . B_q^T)[rows of r] + bias). a (M, K) bf16 (K-major) holds
// every row of this rank's partial product input; b (N, K) (b_kmajor) or (K, N); out (S, N) bf16
// with S = M / world. `recv_peers[q]` is rank q's receive area (two parities of
// `recv_parity_bytes`, each holding world slots of S x N bf16). `pre_out` (S, N) keeps sum + bias.
// `ident` is a 128 x 128 bf16 identity on the device (the B operand that adds received partials).
void tp_gemm_rs(at::Tensor a, at::Tensor b, at::Tensor out, c10::optional<at::Tensor> bias,
                c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> residual,
                c10::optional<at::Tensor> pre_out, bool b_kmajor, std::vector<int64_t> flag_peers,
                std::vector<int64_t> recv_peers, int64_t recv_parity_bytes, int64_t rank, double timeout_ms,
                at::Tensor ident) {
  using namespace tp;
  const int world = (int)flag_peers.size();
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.dim() == 2 && a.is_contiguous(),
              "tp_gemm_rs: a must be a contiguous bf16 (M, K) CUDA matrix");
  const int64_t M = a.size(0), K = a.size(1);
  TORCH_CHECK(M % world == 0, "tp_gemm_rs: M must be divisible by the world size");
  const int64_t S = M / world;
  TORCH_CHECK(world == 1 || S % 128 == 0,
              "tp_gemm_rs: with peers, every rank's row count must be a multiple of 128 (pad the tokens)");
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
  TORCH_CHECK(ident.is_cuda() && ident.scalar_type() == at::kBFloat16 && ident.is_contiguous() && ident.dim() == 2 &&
                  ident.size(0) == kRsBN && ident.size(1) == kRsBN && al16(ident.data_ptr()),
              "tp_gemm_rs: ident must be a contiguous bf16 128 x 128 identity on the device");
  c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  RsParams prm{};
  prm.s = TpShape{(int)M, (int)N, (int)K, (int)S, (int)rank, world, (int)((M + 127) / 128)};
  prm.err = error_word(device);
  const Peers recv = to_peers(recv_peers, world, "tp_gemm_rs recv");
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
  prm.fold_residual = prm.residual != nullptr && prm.gamma == nullptr && prm.pre_out == nullptr;
  prm.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms * 1e6 : 5e9);
  prm.trace = trace_buffer(device, 1);
  RsMaps maps{};
  for (int q = 0; q < world; ++q) {
    const cuuint64_t dims[4] = {(cuuint64_t)N, (cuuint64_t)S, (cuuint64_t)world, 2};
    const cuuint64_t strides[3] = {(cuuint64_t)(N * 2), (cuuint64_t)(S * N * 2), (cuuint64_t)recv_parity_bytes};
    maps.recv[q] = area_map(recv.p[q], 4, dims, strides, "receive slots");
  }
  maps.ident = b_kmajor ? make_bf16_map(ident.data_ptr(), kRsBN, kRsBN, kRsBN, 64, kRsBN)
                        : make_bf16_map(ident.data_ptr(), kRsBN, kRsBN, kRsBN, 64, 64);
  if (prm.fold_residual) maps.res = make_bf16_map(prm.residual, N, S, N, 64, kBM);
  const int64_t tiles = prm.s.num_blocks * ((N + kRsBN - 1) / kRsBN);
  const int grid = (int)std::min<int64_t>(tiles, sm_count(device));
  CUtensorMap ta = make_bf16_map(a.data_ptr(), K, M, K, 64, kBM);
  CUtensorMap tb =
      b_kmajor ? make_bf16_map(b.data_ptr(), K, N, K, 64, kRsBN) : make_bf16_map(b.data_ptr(), N, K, N, 64, 64);
  if (b_kmajor) launch_rs<false>(ta, tb, maps, prm, grid, stream, device);
  else launch_rs<true>(ta, tb, maps, prm, grid, stream, device);
}

int64_t tp_flag_bytes() { return tp::flag_bytes(); }

// (2, ctas, points) int64 CPU tensor: the per-CTA timelines of the last all-gather and reduce-scatter
// launches on `device` (all zero unless MIA_TP_TRACE=1).
at::Tensor tp_trace_read(int64_t device) {
  using namespace tp;
  auto out = at::zeros({2, kTraceCtas, kTracePoints}, at::kLong);
  long long* buf = trace_buffer((int)device, 0);
  if (buf != nullptr) {
    c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
    C10_CUDA_CHECK(cudaDeviceSynchronize());
    C10_CUDA_CHECK(cudaMemcpy(out.data_ptr(), buf, out.numel() * sizeof(long long), cudaMemcpyDeviceToHost));
  }
  return out;
}

}  // namespace mia
