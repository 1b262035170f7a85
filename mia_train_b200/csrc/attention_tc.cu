// Non-causal attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), head dims 32
// and 64, forward and backward.
//
// Forward: one CTA owns 128 queries of one (batch, head) and streams the keys in blocks of 128.
//   warp 0      TMA producer: Q once, K blocks into a 2-deep ring, V blocks into a 1-deep slot.
//               Q / K / V are 4-D tensor maps over strided (D, N, H, B) views, so the kernel reads
//               q / k / v straight out of the packed projection (B, N, 3, H, D) or the rotated
//               buffer (B, N, 2, H, D); rows past N are zero-filled by the TMA unit.
//   warp 1      MMA issuer (one thread): S = Q K^T into TMEM columns [0, 128) (M = 128, N = 128,
//               K = D), then O_j = P_j V_j into TMEM columns [128, 128 + D) (K = 128 keys, V read
//               as an MN-major operand).
//   warps 2-5   softmax: thread = query row = TMEM lane. Reads its S row from TMEM twice (row max,
//               then exp2 + row sum), writes P_j as bf16 into shared memory in the 128-byte
//               swizzled K-major layout the MMA reads, and folds the previous block's O_j from
//               TMEM into a register accumulator with the online-softmax correction.
// Rows are swizzled with the row width (64 B for D = 32, 128 B for D = 64) in both the tensor maps
// and the MMA descriptors. Two forward CTAs fit on an SM (256 TMEM columns, <= 97 KB of shared
// memory each), so one CTA's softmax overlaps the other's MMAs.
//
// Output: o (B, N, H, D) bf16 and the log2-domain row statistic lse = m + log2(l) (B, H, N), the
// same contract as the warp-level kernels in attention.cu; either backward consumes them.
// Every wait is bounded (see common.cuh): on expiry the kernel records kErrAttnWait, lets its own
// copies and MMAs land, frees its tensor memory and returns. Waits are made warp-uniform before
// any `.sync.aligned` TMEM access, and no named (unbounded) barrier is used.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "attention_tc.h"
#include "common.cuh"
#include "errors.h"

namespace mia {
namespace {

typedef __nv_bfloat16 bf16;
constexpr int kTcBM = 128;  // queries per forward CTA
constexpr int kTcBN = 128;  // keys per forward block
constexpr int kTcSoftmaxThreads = 256;  // two warps per TMEM lane quarter, one per half of the keys
constexpr int kTcThreads = 64 + kTcSoftmaxThreads;
constexpr int kBwdSoftmaxThreads = 256;  // two warps per TMEM lane quarter, one per half of the columns
constexpr int kBwdThreads = 64 + kBwdSoftmaxThreads;
constexpr uint32_t kTcTmemCols = 256;

template <int D>
struct TcFwdSmem {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kQBytes = kTcBM * kRowBytes;
  static constexpr int kKVBytes = kTcBN * kRowBytes;
  static constexpr int kPBytes = kTcBM * kTcBN * 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;       // [2]
  static constexpr int kV = kK + 2 * kKVBytes;  // [1]
  static constexpr int kP = kV + kKVBytes;
  static constexpr int kStat = kP + kPBytes;  // (m, l) of both key halves per query row, merged at the end
  static constexpr int kBar = kStat + 4 * kTcBM * 4;
  static constexpr int kBytes = kBar + 128 + 1024;  // barriers, TMEM slot, abort flag, merge counter; slack
};

// All lanes of a warp agree on a bounded wait, so `.sync.aligned` TMEM loads stay warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, kErrAttnWait);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float fast_exp2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, optionally used for a quarter of the softmax exponentials so the
// multi-function unit (16 results per clock per SM) and the FMA pipe share the work.
// Range reduction x = n + f with n = floor(x), f in [0, 1); 2^f by a cubic fitted here to minimise
// the relative error on [0, 1) (iteratively reweighted least squares over 20001 points): maximum
// relative error 7.6e-5, far below the bf16 rounding (3.9e-3) that P is stored with; 2^n is added to
// the exponent field. Arguments below -125 return 0 (the softmax exponents here are <= 0).
__device__ __forceinline__ float poly_exp2f(float x) {
  const float fl = floorf(x);
  const float f = x - fl;
  const float p = fmaf(fmaf(fmaf(0.07802251590f, f, 0.2260656115f), f, 0.6958365058f), f, 0.9999246655f);
  const float y = __int_as_float(__float_as_int(p) + ((int)fl << 23));
  return x < -125.f ? 0.f : y;
}

template <int D, bool kPoly>
__global__ void __launch_bounds__(kTcThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, bf16* __restrict__ o, float* __restrict__ lse, int H,
                       int Nq, int Nk, int q_tiles, float scale_log2, int* err) {
  using L = TcFwdSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;   // [2]
  uint64_t* k_empty = bar + 3;  // [2]
  uint64_t* v_full = bar + 5;
  uint64_t* v_empty = bar + 6;
  uint64_t* s_full = bar + 7;   // S_j in TMEM
  uint64_t* o_full = bar + 8;   // O_j in TMEM (P_j and V_j consumed)
  uint64_t* p_full = bar + 9;   // S_j read, P_j in smem, O_{j-1} read (all softmax threads)
  uint64_t* drain = bar + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q_tile = blockIdx.x % q_tiles;
  const int bh = blockIdx.x / q_tiles;
  const int b = bh / H, h = bh % H;
  const int q0 = q_tile * kTcBM;
  const int nb = (Nk + kTcBN - 1) / kTcBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(o_full, 1);
    mbar_init(p_full, kTcSoftmaxThreads);
    mbar_init(drain, 1);
    *abort_flag = 0;
    tmem_slot[2] = 0;  // softmax warps done (merge counter)
    fence_barrier_init();
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem;
  const uint32_t t_o = tmem + kTcBN;  // O of keys 0..63 of every block; O of keys 64..127 at t_o + D

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, L::kQBytes);
      tma_load_4d(smem + L::kQ, &tmQ, q_full, 0, q0, h, b);
      for (int j = 0; j < nb; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[s], L::kKVBytes);
        tma_load_4d(smem + L::kK + s * L::kKVBytes, &tmK, &k_full[s], 0, j * kTcBN, h, b);
        ++k_issued;
        if (!mbar_wait(v_empty, (j & 1) ^ 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(v_full, L::kKVBytes);
        tma_load_4d(smem + L::kV, &tmV, v_full, 0, j * kTcBN, h, b);
        ++v_issued;
      }
      if (!ok) {
        // Let this CTA's copies in flight land before its shared memory is released.
        mbar_wait(q_full, 0, nullptr, nullptr, 0);
        for (int j = k_issued - 1; j >= 0 && j >= k_issued - 2; --j)
          mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, nullptr, 0);
        if (v_issued > 0) mbar_wait(v_full, (v_issued - 1) & 1, nullptr, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = make_idesc_bf16(kTcBM, kTcBN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kTcBM, D, false, true);
      constexpr uint32_t kSbo = 8 * L::kRowBytes;  // 8-row swizzle atom
      const uint32_t q_addr = smem_u32(smem + L::kQ);
      const uint32_t p_addr = smem_u32(smem + L::kP);
      const uint32_t v_addr = smem_u32(smem + L::kV);
      bool any = false;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, err, kErrAttnWait)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kK + s * L::kKVBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          tc_mma_f16(t_s, make_sdesc_sw<L::kRowBytes>(q_addr + kk * 32, 16, kSbo),
                     make_sdesc_sw<L::kRowBytes>(k_addr + kk * 32, 16, kSbo), idesc_s, kk > 0 ? 1u : 0u);
        }
        any = true;
        tc_commit(&k_empty[s]);
        tc_commit(s_full);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrAttnWait) && issue_s(0);
      for (int j = 0; j < nb && ok; ++j) {
        if (!mbar_wait(p_full, j & 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (j + 1 < nb && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(v_full, j & 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTcBN / 16; ++kk) {
          // A = P (128 x 128 keys, K-major, two 64-key column blocks of 16 KB); B = V (keys x D,
          // D contiguous: MN-major, 16 keys = 16 rows per step).
          // keys 0..63 of the block accumulate into O_0, keys 64..127 into O_1 (each half of the
          // softmax warps keeps its own running maximum and sum; they are merged at the end)
          const uint32_t t_dst = t_o + (kk >> 2) * D;
          tc_mma_f16(t_dst, make_sdesc_sw<128>(p_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                     make_sdesc_sw<L::kRowBytes>(v_addr + kk * 16 * L::kRowBytes, L::kKVBytes, kSbo), idesc_o,
                     (j > 0 || (kk & 3) > 0) ? 1u : 0u);
        }
        tc_commit(v_empty);
        tc_commit(o_full);
      }
      if (!ok && any) {
        tc_commit(drain);
        mbar_wait(drain, 0, nullptr, nullptr, 0);
      }
    }
  } else {
    // -------------------------------------------------------------------- softmax warps
    // Warps 2..9: lane quarter lg = warp & 3, key half `half` = (warp - 2) / 4 (keys 64 * half ..
    // +63 of every block). The two halves of a row are two independent online softmaxes over
    // disjoint keys, each with its own O accumulator in TMEM (O_half), reference maximum and sum;
    // they are merged once at the end. O accumulates over all key blocks (the PV MMAs accumulate),
    // relative to the reference maximum m_ref: P = exp2(s - m_ref) is used as long as a block's
    // maximum stays within kRescale (log2 units) of m_ref, so P <= 2^kRescale; past that the half's
    // O (once the previous PV MMA has landed) and l are scaled by exp2(m_old - m_new) in TMEM.
    constexpr float kRescale = 8.f;
    const int lg = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;
    const int r = lg * 32 + lane;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    const uint32_t t_oh = t_o + half * D;
    uint8_t* P = smem + L::kP;
    float* stat = reinterpret_cast<float*>(smem + L::kStat);  // [2][2][128]: (m, l) of each half
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      if (!warp_wait(s_full, j & 1, abort_flag, err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kbase = j * kTcBN + half * 64;
      // Full key blocks skip the per-element key mask (only the last block can be ragged).
      auto softmax_block = [&](auto full_tag) -> bool {
        constexpr bool kFull = decltype(full_tag)::value;
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_s + lane_off + half * 64 + c * 32, v);
          tmem_ld_wait_regs(v);
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (kFull || kbase + c * 32 + e < Nk) mx = fmaxf(mx, __uint_as_float(v[e]));
        }
        const float blk = mx * scale_log2;
        const bool move = blk > m + kRescale;  // always true for the first block with a key (m = -inf)
        if (__any_sync(0xffffffffu, move && m != -INFINITY)) {
          // rescale this half's O: every PV MMA issued so far has landed once o_full of block j - 1 completes
          if (!warp_wait(o_full, (j - 1) & 1, abort_flag, err)) return false;
          tc_fence_after();
          const float alpha = (move && m != -INFINITY) ? fast_exp2f(m - blk) : 1.f;
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t v[16];
            tmem_ld_32x32b_x16(t_oh + lane_off + c * 16, v);
            tmem_ld_wait_regs16(v);
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st_32x32b_x16(t_oh + lane_off + c * 16, v);
          }
          tmem_st_wait();
          l *= alpha;
        }
        if (move) m = blk;
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_s + lane_off + half * 64 + c * 32, v);
          tmem_ld_wait_regs(v);
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int key = kbase + c * 32 + 2 * e;
            const float p0 =
                (kFull || key < Nk) ? fast_exp2f(fmaf(__uint_as_float(v[2 * e]), scale_log2, -m)) : 0.f;
            const float x1 = fmaf(__uint_as_float(v[2 * e + 1]), scale_log2, -m);
            const float p1 = (kFull || key + 1 < Nk) ? ((!kPoly || (e & 1)) ? fast_exp2f(x1) : poly_exp2f(x1)) : 0.f;
            rs += p0 + p1;
            pk[e] = pack_bf16x2(p0, p1);
          }
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            const int ci = c * 4 + qd;  // 16-byte chunk within the 128-byte row of this half's key block
            uint4* dst = reinterpret_cast<uint4*>(P + half * 16384 + r * 128 + ((ci ^ (r & 7)) << 4));
            *dst = make_uint4(pk[4 * qd], pk[4 * qd + 1], pk[4 * qd + 2], pk[4 * qd + 3]);
          }
        }
        l += rs;
        return true;
      };
      // A half whose keys all lie past Nk (a ragged last block) still writes its zero P.
      const bool done =
          (j * kTcBN + kTcBN <= Nk) ? softmax_block(std::true_type{}) : softmax_block(std::false_type{});
      if (!done) {
        ok = false;
        break;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nb > 0 && !warp_wait(o_full, (nb - 1) & 1, abort_flag, err)) ok = false;
    // merge the two halves: each publishes (m, l) of its rows, then writes half of the output columns
    if (ok) {
      stat[(half * 2 + 0) * 128 + r] = m;
      stat[(half * 2 + 1) * 128 + r] = l;
    }
    __threadfence_block();
    __syncwarp();
    if (lane == 0) atomicAdd(reinterpret_cast<int*>(tmem_slot + 2), ok ? 1 : 1000);
    {
      const uint64_t t0 = globaltimer_ns();
      volatile int* cnt = reinterpret_cast<volatile int*>(tmem_slot + 2);
      while (*cnt < kTcSoftmaxThreads / 32) {
        if (*abort_flag || globaltimer_ns() - t0 > MIA_WAIT_LIMIT_NS) {
          ok = false;
          break;
        }
      }
      ok = __all_sync(0xffffffffu, ok && *cnt < 1000);
    }
    const int qi = q0 + r;
    if (ok && nb > 0) {
      tc_fence_after();
      const float m0 = stat[0 * 128 + r], l0 = stat[1 * 128 + r];
      const float m1 = stat[2 * 128 + r], l1 = stat[3 * 128 + r];
      const float mm = fmaxf(m0, m1);
      const float w0 = m0 == -INFINITY ? 0.f : fast_exp2f(m0 - mm);
      const float w1 = m1 == -INFINITY ? 0.f : fast_exp2f(m1 - mm);
      const float lt = l0 * w0 + l1 * w1;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float a0 = w0 * inv, a1 = w1 * inv;
      bf16* orow = o + (((size_t)b * Nq + (qi < Nq ? qi : 0)) * H + h) * D + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {  // this half's D / 2 output columns, 16 at a time
        uint32_t v0[16], v1[16];
        tmem_ld_32x32b_x16(t_o + lane_off + half * (D / 2) + c * 16, v0);
        tmem_ld_32x32b_x16(t_o + D + lane_off + half * (D / 2) + c * 16, v1);
        tmem_ld_wait_regs16(v0);
        tmem_ld_wait_regs16(v1);
        if (qi < Nq) {
#pragma unroll
          for (int d = 0; d < 16; d += 8) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v0[d + e]) * a0 + __uint_as_float(v1[d + e]) * a1;
            *reinterpret_cast<uint4*>(orow + c * 16 + d) = make_uint4(
                pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          }
        }
      }
      if (qi < Nq && half == 0) lse[(size_t)bh * Nq + qi] = mm + log2f(fmaxf(lt, 1e-30f));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

// ------------------------------------------------------------------------------------ backward
// One CTA owns 128 keys of one (batch, head) and streams the queries in blocks of 128:
//   warp 0      TMA producer: K and V once, then (Q_i, dO_i) into a 2-deep ring.
//   warp 1      MMA issuer: S^T = K Q_i^T and dP^T = V dO_i^T (M = 128 keys, N = 128 queries,
//               K = D) into TMEM; after the softmax warps have written P^T and dS^T to shared memory:
//               dV += P^T dO_i, dK += dS^T Q_i (accumulated in TMEM over all query blocks) and
//               dQ_i = dS K (dS^T read as an MN-major operand).
//   warps 2-9   thread = key row (two warps per row, one per half of the block's queries):
//               P^T = exp2(S^T * scale_log2 - lse_q), dS^T = P^T (dP^T - delta_q) into
//               double-buffered shared memory (128-byte swizzled, K-major over queries); then the
//               previous block's dQ rows (thread = query row, half of the columns) from TMEM into
//               the fp32 dQ buffer with vector atomics; at the end dK and dV rows as bf16.
// TMEM columns: S^T [0, 128), dP^T [128, 256), dV, dK, dQ (D each) from 256; 1 CTA per SM.
// The softmax of block i + 1 overlaps the dV / dK / dQ MMAs of block i. Queries past Nq read
// zero Q / dO rows and lse = +inf, so they contribute nothing; keys past Nk are not stored.
template <int D>
struct TcBwdSmem {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileBytes = 128 * kRowBytes;
  static constexpr int kPBytes = 128 * 128 * 2;
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTileBytes;
  static constexpr int kQ = kV + kTileBytes;       // [2]
  static constexpr int kDO = kQ + 2 * kTileBytes;  // [2]
  static constexpr int kP = kDO + 2 * kTileBytes;  // [2] P^T
  static constexpr int kDS = kP + 2 * kPBytes;     // [2] dS^T
  static constexpr int kStat = kDS + 2 * kPBytes;  // lse[128], delta[128] of the current query block
  static constexpr int kBar = kStat + 1024;
  static constexpr int kBytes = kBar + 160 + 1024;
};

template <int D, bool kPoly>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dq_acc,
                       Strides3 dqs, bf16* __restrict__ dk, Strides3 dks, bf16* __restrict__ dv, Strides3 dvs, int H,
                       int Nq, int Nk, int k_tiles, float scale, float scale_log2, int* err) {
  using L = TcBwdSmem<D>;
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = bar;
  uint64_t* qd_full = bar + 1;     // [2]
  uint64_t* qd_empty = bar + 3;    // [2]
  uint64_t* sdp_full = bar + 5;    // S^T_i and dP^T_i in TMEM
  uint64_t* pds_full = bar + 6;    // S / dP read, P^T / dS^T written (softmax threads)
  uint64_t* buf_free = bar + 7;    // [2] MMAs reading P / dS buffer b completed
  uint64_t* dq_full = bar + 9;     // dQ_i in TMEM (and every earlier MMA complete)
  uint64_t* dq_free = bar + 10;    // dQ_i read (softmax threads)
  uint64_t* drain = bar + 11;
  uint64_t* stat_full = bar + 12;  // lse / delta of the current block in smem (softmax threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_lse = reinterpret_cast<float*>(smem + L::kStat);
  float* s_delta = s_lse + 128;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int k_tile = blockIdx.x % k_tiles;
  const int bh = blockIdx.x / k_tiles;
  const int b = bh / H, h = bh % H;
  const int k0 = k_tile * 128;
  const int nq = (Nq + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
      mbar_init(&buf_free[s], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(pds_full, kBwdSoftmaxThreads);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kBwdSoftmaxThreads);
    mbar_init(drain, 1);
    mbar_init(stat_full, kBwdSoftmaxThreads);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 256 + D, t_dq = tmem + 256 + 2 * D;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      int issued = 0;
      bool ok = true;
      mbar_arrive_expect_tx(kv_full, 2 * L::kTileBytes);
      tma_load_4d(smem + L::kK, &tmK, kv_full, 0, k0, h, b);
      tma_load_4d(smem + L::kV, &tmV, kv_full, 0, k0, h, b);
      for (int i = 0; i < nq; ++i) {
        const int s = i & 1;
        if (!mbar_wait(&qd_empty[s], ((i >> 1) & 1) ^ 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&qd_full[s], 2 * L::kTileBytes);
        tma_load_4d(smem + L::kQ + s * L::kTileBytes, &tmQ, &qd_full[s], 0, i * 128, h, b);
        tma_load_4d(smem + L::kDO + s * L::kTileBytes, &tmDO, &qd_full[s], 0, i * 128, h, b);
        ++issued;
      }
      if (!ok) {
        mbar_wait(kv_full, 0, nullptr, nullptr, 0);
        for (int i = issued - 1; i >= 0 && i >= issued - 2; --i)
          mbar_wait(&qd_full[i & 1], (i >> 1) & 1, nullptr, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_kv = make_idesc_bf16(128, D, false, true);  // dV, dK: A = P^T / dS^T, B = dO / Q
      constexpr uint32_t idesc_q = make_idesc_bf16(128, D, true, true);    // dQ: A = dS (MN-major), B = K
      constexpr uint32_t kSbo = 8 * L::kRowBytes;
      const uint32_t k_addr = smem_u32(smem + L::kK), v_addr = smem_u32(smem + L::kV);
      bool any = false;
      auto issue_sdp = [&](int i) -> bool {
        const int s = i & 1;
        if (!mbar_wait(&qd_full[s], (i >> 1) & 1, abort_flag, err, kErrAttnWait)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + L::kQ + s * L::kTileBytes);
        const uint32_t do_addr = smem_u32(smem + L::kDO + s * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_f16(t_s, make_sdesc_sw<L::kRowBytes>(k_addr + kk * 32, 16, kSbo),
                     make_sdesc_sw<L::kRowBytes>(q_addr + kk * 32, 16, kSbo), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_f16(t_dp, make_sdesc_sw<L::kRowBytes>(v_addr + kk * 32, 16, kSbo),
                     make_sdesc_sw<L::kRowBytes>(do_addr + kk * 32, 16, kSbo), idesc_s, kk > 0 ? 1u : 0u);
        any = true;
        tc_commit(sdp_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, err, kErrAttnWait) && issue_sdp(0);
      for (int i = 0; i < nq && ok; ++i) {
        const int s = i & 1;
        if (!mbar_wait(pds_full, i & 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (i + 1 < nq && !issue_sdp(i + 1)) {
          ok = false;
          break;
        }
        const uint32_t q_addr = smem_u32(smem + L::kQ + s * L::kTileBytes);
        const uint32_t do_addr = smem_u32(smem + L::kDO + s * L::kTileBytes);
        const uint32_t p_addr = smem_u32(smem + L::kP + s * L::kPBytes);
        const uint32_t ds_addr = smem_u32(smem + L::kDS + s * L::kPBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 16 queries per step
          const uint32_t a_off = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t b_off = kk * 16 * L::kRowBytes;
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          tc_mma_f16(t_dv, make_sdesc_sw<128>(p_addr + a_off, 16, 1024),
                     make_sdesc_sw<L::kRowBytes>(do_addr + b_off, L::kTileBytes, kSbo), idesc_kv, acc);
          tc_mma_f16(t_dk, make_sdesc_sw<128>(ds_addr + a_off, 16, 1024),
                     make_sdesc_sw<L::kRowBytes>(q_addr + b_off, L::kTileBytes, kSbo), idesc_kv, acc);
        }
        if (i > 0 && !mbar_wait(dq_free, (i - 1) & 1, abort_flag, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 16 keys per step: dS^T rows kk*16.., K rows kk*16..
          tc_mma_f16(t_dq, make_sdesc_sw<128>(ds_addr + kk * 2048, 16384, 1024),
                     make_sdesc_sw<L::kRowBytes>(k_addr + kk * 16 * L::kRowBytes, L::kTileBytes, kSbo), idesc_q,
                     kk > 0 ? 1u : 0u);
        }
        tc_commit(&qd_empty[s]);
        tc_commit(&buf_free[s]);
        tc_commit(dq_full);
      }
      if (!ok && any) {
        tc_commit(drain);
        mbar_wait(drain, 0, nullptr, nullptr, 0);
      }
    }
  } else {
    // -------------------------------------------------------------------- softmax / epilogue warps
    // Warps 2..9: lane quarter lg = warp & 3 (the TMEM lanes the warp may read), column half
    // `half` = (warp - 2) / 4: queries 64 * half .. +63 of a block (P / dS column block `half`),
    // and columns D / 2 * half .. of dQ / dK / dV.
    const int lg = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = lg * 32 + lane;  // key row (S^T, dP^T, dK, dV) or query row (dQ)
    const int st = threadIdx.x - 64;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    constexpr int kHalfD = D / 2;
    // One statistic per thread: threads 0..127 hold lse, 128..255 delta, of query st % 128.
    const float* stat_src = (st < 128 ? lse : delta) + (size_t)bh * Nq;
    const float stat_pad = st < 128 ? INFINITY : 0.f;
    auto load_stat = [&](int i) -> float {
      const int q = i * 128 + (st & 127);
      return (i < nq && q < Nq) ? stat_src[q] : stat_pad;
    };
    auto dq_epilogue = [&](int i) -> bool {
      if (!warp_wait(dq_full, i & 1, abort_flag, err)) return false;
      tc_fence_after();
      const int qi = i * 128 + r;
      float* dst = dq_acc + (size_t)b * dqs.b + (size_t)h * dqs.h + (size_t)(qi < Nq ? qi : 0) * dqs.n + half * kHalfD;
#pragma unroll
      for (int c = 0; c < kHalfD / 16; ++c) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(t_dq + lane_off + half * kHalfD + c * 16, v);
        tmem_ld_wait_regs16(v);
        if (qi < Nq) {
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            atomicAdd(reinterpret_cast<float4*>(dst + c * 16 + e),
                      make_float4(__uint_as_float(v[e]) * scale, __uint_as_float(v[e + 1]) * scale,
                                  __uint_as_float(v[e + 2]) * scale, __uint_as_float(v[e + 3]) * scale));
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
      return true;
    };
    bool ok = true;
    float stat_next = load_stat(0);
    for (int i = 0; i < nq; ++i) {
      const int s = i & 1;
      // Statistics of block i go to shared memory only after every softmax thread has finished
      // block i - 1, which the completed phase i - 1 of pds_full shows (each thread arrives there
      // after its last read); block i + 1's value is fetched now, off the critical path.
      if (i > 0 && !warp_wait(pds_full, (i - 1) & 1, abort_flag, err)) {
        ok = false;
        break;
      }
      (st < 128 ? s_lse : s_delta)[st & 127] = stat_next;
      stat_next = load_stat(i + 1);
      mbar_arrive(stat_full);
      if (!warp_wait(stat_full, i & 1, abort_flag, err)) {
        ok = false;
        break;
      }
      if (!warp_wait(sdp_full, i & 1, abort_flag, err)) {
        ok = false;
        break;
      }
      if (i >= 2 && !warp_wait(&buf_free[s], ((i - 2) >> 1) & 1, abort_flag, err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint8_t* P = smem + L::kP + s * L::kPBytes + half * 16384;
      uint8_t* DS = smem + L::kDS + s * L::kPBytes + half * 16384;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {  // 32 queries per chunk
        const int c = half * 2 + cc;
        uint32_t sv[32], dpv[32];
        tmem_ld_32x32b_x32(t_s + lane_off + c * 32, sv);
        tmem_ld_32x32b_x32(t_dp + lane_off + c * 32, dpv);
        tmem_ld_wait_regs(sv);
        tmem_ld_wait_regs(dpv);
        uint32_t pk[16], dk2[16];
        const float4* l4 = reinterpret_cast<const float4*>(s_lse + c * 32);
        const float4* d4 = reinterpret_cast<const float4*>(s_delta + c * 32);
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) {
          const float4 lq = l4[e4], dq4 = d4[e4];
          const float ls[4] = {lq.x, lq.y, lq.z, lq.w}, ds[4] = {dq4.x, dq4.y, dq4.z, dq4.w};
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int e = e4 * 2 + e2;
            const float p0 = fast_exp2f(fmaf(__uint_as_float(sv[2 * e]), scale_log2, -ls[2 * e2]));
            const float x1 = fmaf(__uint_as_float(sv[2 * e + 1]), scale_log2, -ls[2 * e2 + 1]);
            const float p1 = (!kPoly || e2) ? fast_exp2f(x1) : poly_exp2f(x1);
            const float d0 = p0 * (__uint_as_float(dpv[2 * e]) - ds[2 * e2]);
            const float d1 = p1 * (__uint_as_float(dpv[2 * e + 1]) - ds[2 * e2 + 1]);
            pk[e] = pack_bf16x2(p0, p1);
            dk2[e] = pack_bf16x2(d0, d1);
          }
        }
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int ci = cc * 4 + qd;
          const uint32_t off = r * 128 + ((ci ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(P + off) = make_uint4(pk[4 * qd], pk[4 * qd + 1], pk[4 * qd + 2], pk[4 * qd + 3]);
          *reinterpret_cast<uint4*>(DS + off) =
              make_uint4(dk2[4 * qd], dk2[4 * qd + 1], dk2[4 * qd + 2], dk2[4 * qd + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pds_full);
      if (i > 0 && !dq_epilogue(i - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && nq > 0) ok = dq_epilogue(nq - 1);
    if (ok) {
      // dq_full of the last block follows every MMA of this CTA: dV and dK are final.
      const int key = k0 + r;
      const size_t key_c = (size_t)(key < Nk ? key : 0);
      bf16* dv_row = dv + (size_t)b * dvs.b + (size_t)h * dvs.h + key_c * dvs.n + half * kHalfD;
      bf16* dk_row = dk + (size_t)b * dks.b + (size_t)h * dks.h + key_c * dks.n + half * kHalfD;
#pragma unroll
      for (int c = 0; c < kHalfD / 16; ++c) {
        uint32_t v[16], w[16];
        tmem_ld_32x32b_x16(t_dv + lane_off + half * kHalfD + c * 16, v);
        tmem_ld_32x32b_x16(t_dk + lane_off + half * kHalfD + c * 16, w);
        tmem_ld_wait_regs16(v);
        tmem_ld_wait_regs16(w);
        if (key < Nk) {
#pragma unroll
          for (int e = 0; e < 16; e += 8) {
            *reinterpret_cast<uint4*>(dv_row + c * 16 + e) =
                make_uint4(pack_bf16x2(__uint_as_float(v[e]), __uint_as_float(v[e + 1])),
                           pack_bf16x2(__uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])),
                           pack_bf16x2(__uint_as_float(v[e + 4]), __uint_as_float(v[e + 5])),
                           pack_bf16x2(__uint_as_float(v[e + 6]), __uint_as_float(v[e + 7])));
            *reinterpret_cast<uint4*>(dk_row + c * 16 + e) =
                make_uint4(pack_bf16x2(__uint_as_float(w[e]) * scale, __uint_as_float(w[e + 1]) * scale),
                           pack_bf16x2(__uint_as_float(w[e + 2]) * scale, __uint_as_float(w[e + 3]) * scale),
                           pack_bf16x2(__uint_as_float(w[e + 4]) * scale, __uint_as_float(w[e + 5]) * scale),
                           pack_bf16x2(__uint_as_float(w[e + 6]) * scale, __uint_as_float(w[e + 7]) * scale));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

// 4-D map over a strided (B, H, N, D) view, box = 128 rows of one (b, h), swizzled by row width.
bool make_head_map(CUtensorMap* map, const void* base, int B, int H, int N, int D, Strides3 s) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  if ((s.n * 2) % 16 != 0 || (s.h * 2) % 16 != 0 || (s.b * 2) % 16 != 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(s.n * 2), (cuuint64_t)(s.h * 2), (cuuint64_t)(s.b * 2)};
  cuuint32_t box[4] = {(cuuint32_t)D, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw = D == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = encode_tiled()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

std::atomic<int> g_tc_attention_mode{1};
// 1: a quarter of the softmax exponentials on the FMA pipe (poly_exp2f); 0 (default): all on the
// MUFU unit. Measured on B200 the split is 5-15% slower at every shape tried (512 x 32 to 32768 x 64):
// the FMA pipe is busy with the scaling, packing and row sums already.
std::atomic<int> g_attention_poly_exp{[] {
  const char* v = std::getenv("MIA_ATTN_POLY");
  return v == nullptr ? 0 : std::atoi(v);
}()};
std::atomic<int64_t> g_tc_attention_launches{0};

template <int D, bool kPoly>
void launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, torch::Tensor& o,
                torch::Tensor& lse, int B, int H, int Nq, int Nk, float scale_log2, int device, cudaStream_t stream) {
  using L = TcFwdSmem<D>;
  auto kern = attn_fwd_tc_kernel<D, kPoly>;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  const int q_tiles = (Nq + kTcBM - 1) / kTcBM;
  const long grid = (long)q_tiles * B * H;
  kern<<<(unsigned)grid, kTcThreads, L::kBytes, stream>>>(mq, mk, mv, reinterpret_cast<bf16*>(o.data_ptr()),
                                                          lse.data_ptr<float>(), H, Nq, Nk, q_tiles, scale_log2,
                                                          error_word(device));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int D, bool kPoly>
void launch_bwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                const torch::Tensor& lse, const torch::Tensor& delta, torch::Tensor& dq_acc, Strides3 dqs,
                torch::Tensor& dk, Strides3 dks, torch::Tensor& dv, Strides3 dvs, int B, int H, int Nq, int Nk,
                float scale, int device, cudaStream_t stream) {
  using L = TcBwdSmem<D>;
  static_assert(L::kBytes <= 232448, "backward shared memory exceeds 227 KB");
  auto kern = attn_bwd_tc_kernel<D, kPoly>;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  const int k_tiles = (Nk + 127) / 128;
  const long grid = (long)k_tiles * B * H;
  constexpr float kLog2e = 1.4426950408889634f;
  kern<<<(unsigned)grid, kBwdThreads, L::kBytes, stream>>>(
      mq, mk, mv, mdo, lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(), dqs,
      reinterpret_cast<bf16*>(dk.data_ptr()), dks, reinterpret_cast<bf16*>(dv.data_ptr()), dvs, H, Nq, Nk, k_tiles,
      scale, scale * kLog2e, error_word(device));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

bool attention_fwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, Strides3 qs,
                      Strides3 ks, Strides3 vs, int B, int H, int Nq, int Nk, int D, torch::Tensor& o,
                      torch::Tensor& lse, float scale_log2) {
  if (g_tc_attention_mode.load() == 0 || (D != 32 && D != 64) || Nq <= 0 || Nk <= 0) return false;
  CUtensorMap mq, mk, mv;
  if (!make_head_map(&mq, q.data_ptr(), B, H, Nq, D, qs) || !make_head_map(&mk, k.data_ptr(), B, H, Nk, D, ks) ||
      !make_head_map(&mv, v.data_ptr(), B, H, Nk, D, vs))
    return false;
  const int device = q.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const bool poly = g_attention_poly_exp.load() != 0;
  if (D == 64) {
    if (poly) launch_fwd<64, true>(mq, mk, mv, o, lse, B, H, Nq, Nk, scale_log2, device, stream);
    else launch_fwd<64, false>(mq, mk, mv, o, lse, B, H, Nq, Nk, scale_log2, device, stream);
  } else {
    if (poly) launch_fwd<32, true>(mq, mk, mv, o, lse, B, H, Nq, Nk, scale_log2, device, stream);
    else launch_fwd<32, false>(mq, mk, mv, o, lse, B, H, Nq, Nk, scale_log2, device, stream);
  }
  g_tc_attention_launches.fetch_add(1);
  return true;
}

bool attention_bwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                      const torch::Tensor& dout, Strides3 qs, Strides3 ks, Strides3 vs, Strides3 dos,
                      const torch::Tensor& lse, const torch::Tensor& delta, torch::Tensor& dq_acc, Strides3 dqs,
                      torch::Tensor& dk, Strides3 dks, torch::Tensor& dv, Strides3 dvs, int B, int H, int Nq, int Nk,
                      int D, float scale) {
  if (g_tc_attention_mode.load() == 0 || (D != 32 && D != 64) || Nq <= 0 || Nk <= 0) return false;
  if ((reinterpret_cast<uintptr_t>(dq_acc.data_ptr()) & 15) != 0 || (dqs.n % 4) != 0 || (dqs.h % 4) != 0 ||
      (dqs.b % 4) != 0)
    return false;  // the dQ atomics are 16-byte vectors
  if ((reinterpret_cast<uintptr_t>(dk.data_ptr()) & 15) != 0 || (reinterpret_cast<uintptr_t>(dv.data_ptr()) & 15) != 0 ||
      (dks.n % 8) != 0 || (dks.h % 8) != 0 || (dks.b % 8) != 0 || (dvs.n % 8) != 0 || (dvs.h % 8) != 0 ||
      (dvs.b % 8) != 0)
    return false;
  CUtensorMap mq, mk, mv, mdo;
  if (!make_head_map(&mq, q.data_ptr(), B, H, Nq, D, qs) || !make_head_map(&mk, k.data_ptr(), B, H, Nk, D, ks) ||
      !make_head_map(&mv, v.data_ptr(), B, H, Nk, D, vs) || !make_head_map(&mdo, dout.data_ptr(), B, H, Nq, D, dos))
    return false;
  const int device = q.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const bool poly = g_attention_poly_exp.load() != 0;
#define MIA_BWD(DD, PP) \
  launch_bwd<DD, PP>(mq, mk, mv, mdo, lse, delta, dq_acc, dqs, dk, dks, dv, dvs, B, H, Nq, Nk, scale, device, stream)
  if (D == 64) {
    if (poly) MIA_BWD(64, true);
    else MIA_BWD(64, false);
  } else {
    if (poly) MIA_BWD(32, true);
    else MIA_BWD(32, false);
  }
#undef MIA_BWD
  g_tc_attention_launches.fetch_add(1);
  return true;
}

void set_tc_attention_mode(int64_t mode) { g_tc_attention_mode.store((int)mode); }
int64_t tc_attention_mode() { return g_tc_attention_mode.load(); }
int64_t tc_attention_launches() { return g_tc_attention_launches.load(); }

int64_t set_attention_poly_exp(int64_t mode) { return g_attention_poly_exp.exchange((int)mode); }

}  // namespace mia
