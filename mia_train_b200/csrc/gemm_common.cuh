// Device-side pieces shared by the tcgen05 GEMM kernels (gemm.cu) and the fused tensor-parallel
// collective GEMMs (tp_gemm.cu): tile constants, the parameter block, and the fused epilogue
// (bias / GELU / GELU' / LayerScale / residual / accumulate / split-K) applied to one 32-column
// chunk of one accumulator row. Host helpers for TMA descriptors are defined in gemm.cu.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace mia {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 16;                   // epilogue warps: 4 per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;   // producer warp, MMA warp, epilogue warps
constexpr int kColParts = kEpiWarps / 4;        // the tile's columns are split this many ways
constexpr int kATileBytes = kBM * kBK * 2;  // 16 KB

enum Act : int { kActNone = 0, kActGelu = 1, kActDGelu = 2 };

struct GemmParams {
  int M, N, K;
  void* D;
  int d_fp32;
  const float* bias;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* aux;  // pre-activation input of GELU' (act == kActDGelu)
  __nv_bfloat16* aux_out;    // pre-activation output (act == kActGelu)
  const float* gamma;
  int act;
  int accumulate;
  int num_m_tiles;
  int num_n_tiles;
  int num_tiles;   // num_m_tiles * num_n_tiles * splits
  int splits;      // split-K factor (> 1: partial sums added atomically into an fp32 output)
  int k_blocks_per_split;
  int* err;
  // Optional column sums of exp(acc * colsum_scale) over the tile rows, atomically added into
  // colsum[N] (single-CTA kernel only): the first column reduction of Sinkhorn-Knopp centring,
  // computed while the prototype logits are still in TMEM.
  float* colsum;
  float colsum_scale;
  // Optional second operand pair (single-CTA kernel, both K-major): the K loop continues over
  // K2 more columns of A2 (M x K2) and B2 (N x K2) into the same accumulator, so
  // D = epi(A B^T + A2 B2^T) -- a low-rank (LoRA) delta added inside the base GEMM's TMEM tile.
  int K2;
};

// Adds sum over the warp's 32 rows of exp(v * scale) for the chunk's 32 columns into colsum[n ..
// n + 31]: a 31-shuffle reduce-scatter across the warp leaves column j's sum in lane j (rows past M
// and columns past N contribute 0). All 32 lanes must call it.
__device__ __forceinline__ void colsum_exp_chunk(const GemmParams& p, int m, int n, const uint32_t (&r)[32], int lane) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j)
    v[j] = (m < p.M && n + j < p.N) ? __expf(__uint_as_float(r[j]) * p.colsum_scale) : 0.f;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float keep = upper ? v[i + off] : v[i];
      const float send = upper ? v[i] : v[i + off];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  if (n + lane < p.N) atomicAdd(p.colsum + n + lane, v[0]);
}

// Tile index -> (m tile, n tile, K-split); m fastest so concurrently running CTAs share B tiles.
struct TileCoord {
  int m0, n0, kb_begin, kb_end;
};
__device__ __forceinline__ TileCoord tile_coord(const GemmParams& p, int tile, int bn, int num_k) {
  const int mn = tile % (p.num_m_tiles * p.num_n_tiles);
  const int split = tile / (p.num_m_tiles * p.num_n_tiles);
  TileCoord c;
  c.m0 = (mn % p.num_m_tiles) * 128;
  c.n0 = (mn / p.num_m_tiles) * bn;
  c.kb_begin = split * p.k_blocks_per_split;
  c.kb_end = min(num_k, c.kb_begin + p.k_blocks_per_split);
  return c;
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kBTileBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kBytes = STAGES * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Epilogue variants, fixed at compile time so each kernel carries only the code it runs (the
// all-features epilogue is large enough to thrash the instruction cache of the warps running it):
//   kEpiPlain  bias / LayerScale / residual / fp32 / accumulate / split-K, no activation
//   kEpiGelu   bias + GELU (+ pre-activation store), bf16 out
//   kEpiDGelu  GELU' from the stored pre-activation, bf16 out
//   kEpiAll    everything (single-CTA kernel)
enum Epi : int { kEpiPlain = 0, kEpiGelu = 1, kEpiDGelu = 2, kEpiAll = 3 };

// `side` (when `use_side`): the chunk's 32 bf16 of the GELU' input (kEpiDGelu) or of the residual
// (kEpiPlain), loaded by the caller while its TMEM load is in flight.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int m, int n, const uint32_t (&r)[32],
                                               bool use_side, const uint4 (&side)[4]) {
  if (m >= p.M || n >= p.N) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  constexpr bool kAct = EPI != kEpiPlain;
  constexpr bool kExtras = EPI == kEpiPlain || EPI == kEpiAll;  // LayerScale, residual, fp32, accumulate, split-K
  if (kExtras && p.splits > 1) {  // split-K partial: atomically added into the fp32 output
    float* dst = reinterpret_cast<float*>(p.D) + (size_t)m * p.N + n;
    if (n + 32 <= p.N) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        atomicAdd(reinterpret_cast<float4*>(dst) + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < p.N) atomicAdd(dst + j, v[j]);
    }
    return;
  }
  const bool full = (n + 32 <= p.N);
  const size_t row = (size_t)m * p.N;
  if (p.bias != nullptr) {
    if (full) {
      const float4* b4 = reinterpret_cast<const float4*>(p.bias + n);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 bb = __ldg(b4 + q);
        v[4 * q] += bb.x; v[4 * q + 1] += bb.y; v[4 * q + 2] += bb.z; v[4 * q + 3] += bb.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < p.N) v[j] += __ldg(p.bias + n + j);
    }
  }
  if (kAct && (EPI == kEpiGelu || p.act == kActGelu)) {
    if (p.aux_out != nullptr) {
      if (full) {
        uint4* dst = reinterpret_cast<uint4*>(p.aux_out + row + n);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16x2(v[8 * q + 0], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                              pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n + j < p.N) p.aux_out[row + n + j] = __float2bfloat16_rn(v[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
  } else if (kAct && (EPI == kEpiDGelu || p.act == kActDGelu)) {
    if (full) {
      const uint4* src = reinterpret_cast<const uint4*>(p.aux + row + n);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = use_side ? side[q] : __ldg(src + q);
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * q + 2 * h] *= gelu_erf_grad(bf16_lo(w[h]));
          v[8 * q + 2 * h + 1] *= gelu_erf_grad(bf16_hi(w[h]));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < p.N) v[j] *= gelu_erf_grad(__bfloat162float(p.aux[row + n + j]));
    }
  }
  if (kExtras && p.gamma != nullptr) {
    if (full) {
      const float4* g4 = reinterpret_cast<const float4*>(p.gamma + n);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 gg = __ldg(g4 + q);
        v[4 * q] *= gg.x; v[4 * q + 1] *= gg.y; v[4 * q + 2] *= gg.z; v[4 * q + 3] *= gg.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < p.N) v[j] *= __ldg(p.gamma + n + j);
    }
  }
  if (kExtras && p.residual != nullptr) {
    if (full) {
      const uint4* src = reinterpret_cast<const uint4*>(p.residual + row + n);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = use_side ? side[q] : __ldg(src + q);
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * q + 2 * h] += bf16_lo(w[h]);
          v[8 * q + 2 * h + 1] += bf16_hi(w[h]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < p.N) v[j] += __bfloat162float(p.residual[row + n + j]);
    }
  }
  if (kExtras && p.d_fp32) {
    float* dst = reinterpret_cast<float*>(p.D) + row + n;
    if (full) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        if (p.accumulate) {
          float4 old = d4[q];
          o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
        }
        d4[q] = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < p.N) dst[j] = p.accumulate ? dst[j] + v[j] : v[j];
    }
  } else {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.D) + row + n;
    if (full) {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (kExtras && p.accumulate) {
          uint4 old = d4[q];
          uint32_t w[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            v[8 * q + 2 * h] += bf16_lo(w[h]);
            v[8 * q + 2 * h + 1] += bf16_hi(w[h]);
          }
        }
        d4[q] = make_uint4(pack_bf16x2(v[8 * q + 0], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                           pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (n + j < p.N) {
          const float o = v[j] + ((kExtras && p.accumulate) ? __bfloat162float(dst[j]) : 0.f);
          dst[j] = __float2bfloat16_rn(o);
        }
      }
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int m, int n, const uint32_t (&r)[32]) {
  const uint4 none[4] = {};
  epilogue_chunk<EPI>(p, m, n, r, false, none);
}


// 2-D bf16 tensor map over a row-major (rows x inner) matrix with row stride `ld` elements,
// 128-byte swizzle, box (box_inner x box_rows). Defined in gemm.cu.
CUtensorMap make_bf16_map(const void* base, int64_t inner, int64_t rows, int64_t ld, int box_inner, int box_rows);
int sm_count(int device);

}  // namespace mia
