// Non-causal multi-head attention, forward and backward, plus the RoPE split/merge around it.
//
// Layouts: q, k, v, dq, dk, dv are strided (B, H, N, D) views with contiguous D rows; the output
// o and its gradient do are (B, N, H, D) so the output projection reads them as (B*N, H*D).
//
// Forward (flash-style, one CTA per 64 queries of one (b, h), 4 warps x 16 query rows): K/V
// blocks of 64 keys stream through double-buffered shared memory (cp.async), S = Q K^T and
// O += P V run on warp-level bf16 tensor-core tiles (16x8x16), the softmax is online in the
// exp2 domain. `lse` holds log2-domain row statistics m + log2(l) (internal to this pair of kernels).
//
// Backward (one CTA per 64 keys of one (b, h), 4 warps x 16 keys): loops over query blocks,
// recomputes P^T from lse, accumulates dV and dK in registers, and adds dQ = dS K into an fp32
// buffer with one atomic per element per CTA. `delta = rowsum(dO * O)` is a separate pass.
//
// The kernels take (batch, head, row) element strides, so they read q / k / v straight out of the
// packed projection (B, N, 3, H, D) or the rotated buffer (B, N, 2, H, D) as well as from
// contiguous (B, H, N, D) tensors. RoPE kernels: see the section below.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <utility>

#include "attention_tc.h"
#include "common.cuh"

namespace mia {

typedef __nv_bfloat16 bf16;
constexpr int kAttnBlockM = 64;
constexpr int kAttnBlockN = 64;
constexpr int kAttnThreads = 128;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = smem_u32(smem);
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}


// 2^x with the hardware approximation (relative error ~2^-22, flushes denormals), for softmax terms.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// C(16x8 fp32) += A(16x16 bf16, row) * B(16x8 bf16, col)
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Loads `rows` x D bf16 rows (row stride `ld` elements in global) into padded shared memory.
template <int D>
__device__ __forceinline__ void load_rows_async(bf16* smem, const bf16* g, int64_t ld, int row0, int rows, int nvalid) {
  constexpr int kChunks = D / 8;
  constexpr int kStride = D + 8;
  for (int i = threadIdx.x; i < rows * kChunks; i += blockDim.x) {
    const int r = i / kChunks, c = i % kChunks;
    const bool valid = (row0 + r) < nvalid;
    const bf16* src = g + (size_t)(valid ? row0 + r : 0) * ld + c * 8;
    cp_async16(smem + r * kStride + c * 8, src, valid);
  }
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                                const bf16* __restrict__ v, bf16* __restrict__ o,
                                                                float* __restrict__ lse, int H, int Nq, int Nk,
                                                                float scale_log2, Strides3 qs, Strides3 ks, Strides3 vs) {
  constexpr int S = D + 8;  // padded row stride (elements)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  bf16* Qs = reinterpret_cast<bf16*>(smem_raw);
  bf16* Ks = Qs + kAttnBlockM * S;            // [2][64][S]
  bf16* Vs = Ks + 2 * kAttnBlockN * S;        // [2][64][S]
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kAttnBlockM;
  const bf16* qg = q + b * qs.b + h * qs.h;
  const bf16* kg = k + b * ks.b + h * ks.h;
  const bf16* vg = v + b * vs.b + h * vs.h;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, t = lane % 4;

  load_rows_async<D>(Qs, qg, qs.n, q0, kAttnBlockM, Nq);
  load_rows_async<D>(Ks, kg, ks.n, 0, kAttnBlockN, Nk);
  load_rows_async<D>(Vs, vg, vs.n, 0, kAttnBlockN, Nk);
  cp_async_commit();

  uint32_t qf[D / 16][4];
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  const int n_blocks = (Nk + kAttnBlockN - 1) / kAttnBlockN;
  for (int j = 0; j < n_blocks; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_blocks) {
      load_rows_async<D>(Ks + (buf ^ 1) * kAttnBlockN * S, kg, ks.n, (j + 1) * kAttnBlockN, kAttnBlockN, Nk);
      load_rows_async<D>(Vs + (buf ^ 1) * kAttnBlockN * S, vg, vs.n, (j + 1) * kAttnBlockN, kAttnBlockN, Nk);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int row = warp * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        const int col = kk * 16 + 8 * (lane / 16);
        ldsm_x4(qf[kk], Qs + row * S + col);
      }
    }
    const bf16* Kb = Ks + buf * kAttnBlockN * S;
    const bf16* Vb = Vs + buf * kAttnBlockN * S;
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r[4];
        const int row = np * 16 + (lane % 8) + 8 * (lane / 16);
        const int col = kk * 16 + 8 * ((lane / 8) % 2);
        ldsm_x4(r, Kb + row * S + col);
        mma16816(s[2 * np], qf[kk], r[0], r[1]);
        mma16816(s[2 * np + 1], qf[kk], r[2], r[3]);
      }
    }
    // scale, mask, online softmax
    const int kbase = j * kAttnBlockN;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + nt * 8 + 2 * t + (e & 1);
        float val = s[nt][e] * scale_log2;
        if (key >= Nk) val = -INFINITY;
        s[nt][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      corr[r] = (m_run[r] == -INFINITY) ? 0.f : fast_exp2(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mr = m_run[e >> 1];
        const float p = (s[nt][e] == -INFINITY) ? 0.f : fast_exp2(s[nt][e] - mr);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      acc[dt][0] *= corr[0];
      acc[dt][1] *= corr[0];
      acc[dt][2] *= corr[1];
      acc[dt][3] *= corr[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t r[4];
        const int row = kk * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        const int col = dp * 16 + 8 * (lane / 16);
        ldsm_x4_t(r, Vb + row * S + col);
        mma16816(acc[2 * dp], pa, r[0], r[1]);
        mma16816(acc[2 * dp + 1], pa, r[2], r[3]);
      }
    }
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = q0 + warp * 16 + g + 8 * r;
    if (qi >= Nq) continue;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
    bf16* orow = o + (((size_t)b * Nq + qi) * H + h) * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * t) =
          pack_bf16x2(acc[dt][2 * r] * inv, acc[dt][2 * r + 1] * inv);
    }
    if (t == 0) lse[(size_t)bh * Nq + qi] = m_run[r] + log2f(fmaxf(l_run[r], 1e-30f));
  }
}

// delta[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d]. One thread per (b, i, h) row in memory
// order, so a warp reads 32 consecutive rows with 16-byte loads. When `zero_rows` is given (an
// fp32 (B, N, H, D) buffer, e.g. the dQ accumulator of the backward that follows), the same row of
// it is cleared, which saves a separate fill.
template <int D>
__global__ void attn_delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout, float* __restrict__ delta,
                                  int H, int N, int rows, float* __restrict__ zero_rows = nullptr) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  if (zero_rows != nullptr) {
    float4* z = reinterpret_cast<float4*>(zero_rows + (size_t)row * D);
#pragma unroll
    for (int i = 0; i < D / 4; ++i) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const uint4* a4 = reinterpret_cast<const uint4*>(o + (size_t)row * D);
  const uint4* c4 = reinterpret_cast<const uint4*>(dout + (size_t)row * D);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const uint4 a = a4[i], c = c4[i];
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wc[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) s += bf16_lo(wa[j]) * bf16_lo(wc[j]) + bf16_hi(wa[j]) * bf16_hi(wc[j]);
  }
  const int h = row % H;
  const int bn = row / H;
  const int b = bn / N, i = bn % N;
  delta[((size_t)b * H + h) * N + i] = s;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_bwd_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, const bf16* __restrict__ dout,
    const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dq_acc, bf16* __restrict__ dk,
    bf16* __restrict__ dv, int H, int Nq, int Nk, float scale, float scale_log2, Strides3 qs, Strides3 ks, Strides3 vs,
    Strides3 dqs, Strides3 dks, Strides3 dvs) {
  constexpr int S = D + 8;
  constexpr int SP = kAttnBlockM + 8;  // dS^T row stride
  extern __shared__ __align__(16) uint8_t smem_raw[];
  bf16* Ks = reinterpret_cast<bf16*>(smem_raw);  // [64][S]
  bf16* Vs = Ks + kAttnBlockN * S;               // [64][S]
  bf16* Qs = Vs + kAttnBlockN * S;               // [64][S]
  bf16* dOs = Qs + kAttnBlockM * S;              // [64][S]
  bf16* dSs = dOs + kAttnBlockM * S;             // [64 keys][SP]
  float* lse_s = reinterpret_cast<float*>(dSs + kAttnBlockN * SP);
  float* delta_s = lse_s + kAttnBlockM;

  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int k0 = blockIdx.x * kAttnBlockN;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, t = lane % 4;
  const bf16* qg = q + b * qs.b + h * qs.h;
  const bf16* kg = k + b * ks.b + h * ks.h;
  const bf16* vg = v + b * vs.b + h * vs.h;
  const bf16* dog = dout + ((size_t)b * Nq * H + h) * D;  // row stride H*D

  load_rows_async<D>(Ks, kg, ks.n, k0, kAttnBlockN, Nk);
  load_rows_async<D>(Vs, vg, vs.n, k0, kAttnBlockN, Nk);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  uint32_t kf[D / 16][4], vf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int row = warp * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
    const int col = kk * 16 + 8 * (lane / 16);
    ldsm_x4(kf[kk], Ks + row * S + col);
    ldsm_x4(vf[kk], Vs + row * S + col);
  }
  float dk_acc[D / 8][4], dv_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk_acc[i][e] = dv_acc[i][e] = 0.f;

  const int my_key0 = k0 + warp * 16;
  const int n_qblocks = (Nq + kAttnBlockM - 1) / kAttnBlockM;
  for (int qb = 0; qb < n_qblocks; ++qb) {
    const int q0 = qb * kAttnBlockM;
    load_rows_async<D>(Qs, qg, qs.n, q0, kAttnBlockM, Nq);
    load_rows_async<D>(dOs, dog, (int64_t)H * D, q0, kAttnBlockM, Nq);
    cp_async_commit();
    for (int i = threadIdx.x; i < kAttnBlockM; i += blockDim.x) {
      const int qi = q0 + i;
      lse_s[i] = qi < Nq ? lse[(size_t)bh * Nq + qi] : 0.f;
      delta_s[i] = qi < Nq ? delta[(size_t)bh * Nq + qi] : 0.f;
    }
    cp_async_wait<0>();
    __syncthreads();

    // S^T = K_w Q^T : 16 keys x 64 queries
    float st[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) st[nt][0] = st[nt][1] = st[nt][2] = st[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r[4];
        const int row = np * 16 + (lane % 8) + 8 * (lane / 16);
        const int col = kk * 16 + 8 * ((lane / 8) % 2);
        ldsm_x4(r, Qs + row * S + col);
        mma16816(st[2 * np], kf[kk], r[0], r[1]);
        mma16816(st[2 * np + 1], kf[kk], r[2], r[3]);
      }
    }
    // P^T
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi_local = nt * 8 + 2 * t + (e & 1);
        const int key = my_key0 + g + 8 * (e >> 1);
        const bool valid = (q0 + qi_local < Nq) && (key < Nk);
        st[nt][e] = valid ? fast_exp2(st[nt][e] * scale_log2 - lse_s[qi_local]) : 0.f;
      }
    }
    // dV += P^T dO
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t r[4];
        const int row = kk * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        const int col = dp * 16 + 8 * (lane / 16);
        ldsm_x4_t(r, dOs + row * S + col);
        mma16816(dv_acc[2 * dp], pa, r[0], r[1]);
        mma16816(dv_acc[2 * dp + 1], pa, r[2], r[3]);
      }
    }
    // dP^T = V_w dO^T
    float dpt[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) dpt[nt][0] = dpt[nt][1] = dpt[nt][2] = dpt[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r[4];
        const int row = np * 16 + (lane % 8) + 8 * (lane / 16);
        const int col = kk * 16 + 8 * ((lane / 8) % 2);
        ldsm_x4(r, dOs + row * S + col);
        mma16816(dpt[2 * np], vf[kk], r[0], r[1]);
        mma16816(dpt[2 * np + 1], vf[kk], r[2], r[3]);
      }
    }
    // dS^T = P^T * (dP^T - delta); stash as bf16 for the dQ product
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi_local = nt * 8 + 2 * t + (e & 1);
        st[nt][e] = st[nt][e] * (dpt[nt][e] - delta_s[qi_local]);
      }
      const int krow = warp * 16 + g;
      *reinterpret_cast<uint32_t*>(dSs + krow * SP + nt * 8 + 2 * t) = pack_bf16x2(st[nt][0], st[nt][1]);
      *reinterpret_cast<uint32_t*>(dSs + (krow + 8) * SP + nt * 8 + 2 * t) = pack_bf16x2(st[nt][2], st[nt][3]);
    }
    // dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t r[4];
        const int row = kk * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        const int col = dp * 16 + 8 * (lane / 16);
        ldsm_x4_t(r, Qs + row * S + col);
        mma16816(dk_acc[2 * dp], pa, r[0], r[1]);
        mma16816(dk_acc[2 * dp + 1], pa, r[2], r[3]);
      }
    }
    __syncthreads();
    // dQ (warp's 16 queries x D) = dS (16 q x 64 keys) K (64 keys x D)
    float dq[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16-key slices
      uint32_t a[4];
      {
        // A[q][key] = dSs[key][q]: transposed load. Matrices: (q 0-7, keys 0-7), (q 8-15, keys 0-7),
        // (q 0-7, keys 8-15), (q 8-15, keys 8-15).
        const int mat = lane / 8;
        const int key = kk * 16 + (lane % 8) + 8 * (mat / 2);
        const int qq = warp * 16 + 8 * (mat % 2);
        ldsm_x4_t(a, dSs + key * SP + qq);
      }
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t r[4];
        const int row = kk * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        const int col = dp * 16 + 8 * (lane / 16);
        ldsm_x4_t(r, Ks + row * S + col);
        mma16816(dq[2 * dp], a, r[0], r[1]);
        mma16816(dq[2 * dp + 1], a, r[2], r[3]);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int qi = q0 + warp * 16 + g + 8 * r;
      if (qi >= Nq) continue;
      float* dst = dq_acc + b * dqs.b + h * dqs.h + qi * dqs.n;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt)
        atomicAdd(reinterpret_cast<float2*>(dst + dt * 8 + 2 * t), make_float2(dq[dt][2 * r] * scale, dq[dt][2 * r + 1] * scale));
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = my_key0 + g + 8 * r;
    if (key >= Nk) continue;
    bf16* dkr = dk + b * dks.b + h * dks.h + key * dks.n;
    bf16* dvr = dv + b * dvs.b + h * dvs.h + key * dvs.n;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      *reinterpret_cast<uint32_t*>(dkr + dt * 8 + 2 * t) =
          pack_bf16x2(dk_acc[dt][2 * r] * scale, dk_acc[dt][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(dvr + dt * 8 + 2 * t) = pack_bf16x2(dv_acc[dt][2 * r], dv_acc[dt][2 * r + 1]);
    }
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, size_t n) {
  size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 2;
  if (i + 1 < n) {
    float2 v = *reinterpret_cast<const float2*>(src + i);
    *reinterpret_cast<uint32_t*>(dst + i) = pack_bf16x2(v.x, v.y);
  } else if (i < n) {
    dst[i] = __float2bfloat16_rn(src[i]);
  }
}

// ------------------------------------------------------------------------------------ RoPE
// Token-major RoPE around the attention kernels. The fused projection qkv (B, N, 3, H, D) is never
// split: v is read in place, q and k are rotated into qk (B, N, 2, H, D) by `rope_qk_fwd_kernel`,
// and the attention kernels take strided (B, N, H, D) views. One warp per (token, q|k): the warp
// stages the token's H*D channels in shared memory with 16-byte loads; lane p owns pair p
// (channels i1, i2 of `pairs`, the sine and cosine of the token's angle p in registers) and
// rotates that pair in every head in place; the row is written back with 16-byte stores. Channels
// outside every pair pass through unchanged.
//
// Backward (`rope_qk_bwd_kernel`): the attention backward leaves dq (fp32, token-major) and the
// rotated-space dk in the dqkv slot; the warp un-rotates both into dqkv (B, N, 3, H, D), lane p
// accumulating d(angle_p) = sum_heads (g2 y1 - g1 y2) in a register, and the two warps of a token
// add their parts through shared memory, so the token's angle gradient is written once.
constexpr int kRopeTokensPerCta = 4;  // warps = 2 * tokens

__device__ __forceinline__ size_t rope_fwd_warp_bytes(int HD) { return ((size_t)HD * 2 + 15) / 16 * 16; }
__device__ __forceinline__ size_t rope_bwd_warp_bytes(int HD, int P) {
  return ((size_t)HD * 6 + (size_t)P * 4 + 15) / 16 * 16;
}

// qkv (B, N, 3, H, D) -> qk (B, N, 2, H, D); angles (B or 1, N, P) fp32.
__global__ void rope_qk_fwd_kernel(const bf16* __restrict__ qkv, const float* __restrict__ angles,
                                   const int* __restrict__ pairs, int P, int64_t angle_bstride, bf16* __restrict__ qk,
                                   int BN, int N, int H, int D) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int HD = H * D;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  bf16* xs = reinterpret_cast<bf16*>(smem_raw + warp * rope_fwd_warp_bytes(HD));
  const int token = blockIdx.x * kRopeTokensPerCta + warp / 2;
  const int which = warp % 2;
  if (token >= BN) return;  // no CTA-wide barrier below
  const int b = token / N, n = token % N;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + ((size_t)token * 3 + which) * HD);
#pragma unroll 4
  for (int c = lane; c < HD / 8; c += 32) reinterpret_cast<uint4*>(xs)[c] = src[c];
  const float* ang = angles + (size_t)b * angle_bstride + (size_t)n * P;
  __syncwarp();
  for (int p = lane; p < P; p += 32) {
    const int i1 = pairs[2 * p], i2 = pairs[2 * p + 1];
    float sn, cs;
    sincosf(ang[p], &sn, &cs);
    for (int h = 0; h < H; ++h) {
      bf16* row = xs + h * D;
      const float a = __bfloat162float(row[i1]), c2 = __bfloat162float(row[i2]);
      row[i1] = __float2bfloat16_rn(a * cs - c2 * sn);
      row[i2] = __float2bfloat16_rn(c2 * cs + a * sn);
    }
  }
  __syncwarp();
  uint4* dst = reinterpret_cast<uint4*>(qk + ((size_t)token * 2 + which) * HD);
#pragma unroll 4
  for (int c = lane; c < HD / 8; c += 32) dst[c] = reinterpret_cast<const uint4*>(xs)[c];
}

// dq_acc (B, N, H, D) fp32; dqkv (B, N, 3, H, D) with the rotated-space dk in slot 1 and dv in
// slot 2; y = the rotated q/k the attention saw (`qk`, or qkv itself when P == 0).
__global__ void rope_qk_bwd_kernel(const float* __restrict__ dq_acc, const bf16* __restrict__ y, int64_t y_token_stride,
                                   const float* __restrict__ angles, const int* __restrict__ pairs, int P,
                                   int64_t angle_bstride, bf16* __restrict__ dqkv, float* __restrict__ dangles, int BN,
                                   int N, int H, int D) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int HD = H * D;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const size_t per_warp = rope_bwd_warp_bytes(HD, P);
  uint8_t* base = smem_raw + warp * per_warp;
  float* gs = reinterpret_cast<float*>(base);
  bf16* ys = reinterpret_cast<bf16*>(base + (size_t)HD * 4);
  float* dpart = reinterpret_cast<float*>(base + (size_t)HD * 6);
  const int token = blockIdx.x * kRopeTokensPerCta + warp / 2;
  const int which = warp % 2;
  const bool active = token < BN;
  const int b = active ? token / N : 0, n = active ? token % N : 0;
  bf16* dst = dqkv + ((size_t)token * 3 + which) * HD;
  if (active && !(P == 0 && which == 1)) {  // without RoPE the dk slot is already final
    if (which == 0) {
      const float4* g4 = reinterpret_cast<const float4*>(dq_acc + (size_t)token * HD);
#pragma unroll 4
      for (int c = lane; c < HD / 4; c += 32) reinterpret_cast<float4*>(gs)[c] = g4[c];
    } else {
      const uint4* g8 = reinterpret_cast<const uint4*>(dst);
#pragma unroll 4
      for (int c = lane; c < HD / 8; c += 32) {
        const uint4 u = g8[c];
        reinterpret_cast<float4*>(gs)[2 * c] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
        reinterpret_cast<float4*>(gs)[2 * c + 1] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
      }
    }
    if (P > 0) {
      const uint4* y8 = reinterpret_cast<const uint4*>(y + (size_t)token * y_token_stride + (size_t)which * HD);
#pragma unroll 4
      for (int c = lane; c < HD / 8; c += 32) reinterpret_cast<uint4*>(ys)[c] = y8[c];
      __syncwarp();
      const float* ang = angles + (size_t)b * angle_bstride + (size_t)n * P;
      for (int p = lane; p < P; p += 32) {
        const int i1 = pairs[2 * p], i2 = pairs[2 * p + 1];
        float sn, cs;
        sincosf(ang[p], &sn, &cs);
        float acc = 0.f;
        for (int h = 0; h < H; ++h) {
          float* g = gs + h * D;
          const bf16* yr = ys + h * D;
          const float g1 = g[i1], g2 = g[i2];
          acc += g2 * __bfloat162float(yr[i1]) - g1 * __bfloat162float(yr[i2]);
          // inverse rotation: the transpose of [[c, -s], [s, c]] acting on (first, second)
          g[i1] = g1 * cs + g2 * sn;
          g[i2] = g2 * cs - g1 * sn;
        }
        dpart[p] = acc;
      }
    }
    __syncwarp();
#pragma unroll 4
    for (int c = lane; c < HD / 8; c += 32) {
      const float4 a = reinterpret_cast<const float4*>(gs)[2 * c], e = reinterpret_cast<const float4*>(gs)[2 * c + 1];
      reinterpret_cast<uint4*>(dst)[c] =
          make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(e.x, e.y), pack_bf16x2(e.z, e.w));
    }
  }
  __syncthreads();
  if (active && dangles != nullptr && P > 0 && which == 0) {
    // partner warp (the token's k) is warp + 1, same CTA
    const float* kpart = reinterpret_cast<const float*>(smem_raw + (warp + 1) * per_warp + (size_t)HD * 6);
    for (int p = lane; p < P; p += 32) dangles[(size_t)token * P + p] = dpart[p] + kpart[p];
  }
}

// ------------------------------------------------------------------------------------ host
static constexpr float kLog2e = 1.4426950408889634f;

#define DISPATCH_HEAD_DIM(D_, ...)                                            \
  [&] {                                                                       \
    if ((D_) == 32) { constexpr int HD = 32; return __VA_ARGS__(); }          \
    if ((D_) == 64) { constexpr int HD = 64; return __VA_ARGS__(); }          \
    if ((D_) == 128) { constexpr int HD = 128; return __VA_ARGS__(); }        \
    TORCH_CHECK(false, "attention: head_dim must be 32, 64 or 128, got ", D_); \
  }()

// Strides of a (B, H, N, D) tensor and of a (B, N, H, D) view presented as (B, H, N, D).
static Strides3 bhnd_strides(const torch::Tensor& t) { return Strides3{t.stride(0), t.stride(1), t.stride(2)}; }
static Strides3 bnhd_strides(const torch::Tensor& t) { return Strides3{t.stride(0), t.stride(2), t.stride(1)}; }
// Strides of a contiguous (B, N, H, D) buffer (e.g. dO) presented as (B, H, N, D).
static Strides3 bnhd_contiguous(int N, int H, int D) { return Strides3{(int64_t)N * H * D, D, (int64_t)H * D}; }

void attention_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse, double scale) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "attention_fwd: contiguous bf16 (B, H, N, D) inputs");
  const int B = (int)q.size(0), H = (int)q.size(1), Nq = (int)q.size(2), D = (int)q.size(3);
  const int Nk = (int)k.size(2);
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (Nq == 0) return;
  if (attention_fwd_tc(q, k, v, bhnd_strides(q), bhnd_strides(k), bhnd_strides(v), B, H, Nq, Nk, D, o, lse,
                       (float)scale * kLog2e))
    return;
  DISPATCH_HEAD_DIM(D, [&] {
    constexpr int S = HD + 8;
    const size_t smem = (size_t)(kAttnBlockM + 4 * kAttnBlockN) * S * 2;
    auto kern = attn_fwd_kernel<HD>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((Nq + kAttnBlockM - 1) / kAttnBlockM, B * H);
    kern<<<grid, kAttnThreads, smem, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
        reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), H,
        Nq, Nk, (float)scale * kLog2e, bhnd_strides(q), bhnd_strides(k), bhnd_strides(v));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  });
}

// Runs delta + main backward; dq is written as fp32 into `dq_acc` (B, H, Nq, D) (zeroed here).
static void attention_bwd_core(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                               torch::Tensor lse, torch::Tensor dq_acc, torch::Tensor dk, torch::Tensor dv,
                               double scale) {
  const int B = (int)q.size(0), H = (int)q.size(1), Nq = (int)q.size(2), D = (int)q.size(3);
  const int Nk = (int)k.size(2);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto delta = torch::empty({B, H, Nq}, q.options().dtype(at::kFloat));
  C10_CUDA_CHECK(cudaMemsetAsync(dq_acc.data_ptr(), 0, dq_acc.numel() * 4, stream));
  DISPATCH_HEAD_DIM(D, [&] {
    const int rows = B * H * Nq;
    attn_delta_kernel<HD><<<(rows + 255) / 256, 256, 0, stream>>>(
        reinterpret_cast<const bf16*>(o.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
        delta.data_ptr<float>(), H, Nq, rows);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    if (attention_bwd_tc(q, k, v, dout, bhnd_strides(q), bhnd_strides(k), bhnd_strides(v), bnhd_contiguous(Nq, H, D),
                         lse, delta, dq_acc, bhnd_strides(dq_acc), dk, bhnd_strides(dk), dv, bhnd_strides(dv), B, H,
                         Nq, Nk, D, (float)scale))
      return;
    constexpr int S = HD + 8;
    const size_t smem = (size_t)(2 * kAttnBlockN + 2 * kAttnBlockM) * S * 2 + (size_t)kAttnBlockN * (kAttnBlockM + 8) * 2 +
                        2 * kAttnBlockM * 4;
    auto kern = attn_bwd_kernel<HD>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((Nk + kAttnBlockN - 1) / kAttnBlockN, B * H);
    kern<<<grid, kAttnThreads, smem, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
        reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
        lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
        reinterpret_cast<bf16*>(dk.data_ptr()), reinterpret_cast<bf16*>(dv.data_ptr()), H, Nq, Nk, (float)scale,
        (float)scale * kLog2e, bhnd_strides(q), bhnd_strides(k), bhnd_strides(v), bhnd_strides(dq_acc),
        bhnd_strides(dk), bhnd_strides(dv));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  });
}

void attention_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                   torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(dout.is_contiguous() && o.is_contiguous(), "attention_bwd: contiguous o / do");
  auto dq_acc = torch::empty(q.sizes(), q.options().dtype(at::kFloat));
  attention_bwd_core(q, k, v, o, dout, lse, dq_acc, dk, dv, scale);
  const size_t n = dq.numel();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  f32_to_bf16_kernel<<<(unsigned)((n / 2 + 255) / 256 + 1), 256, 0, stream>>>(dq_acc.data_ptr<float>(),
                                                                              reinterpret_cast<bf16*>(dq.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static size_t rope_fwd_smem(int H, int D, int P) {
  (void)P;
  return ((size_t)H * D * 2 + 15) / 16 * 16 * 2 * kRopeTokensPerCta;
}

static size_t rope_bwd_smem(int H, int D, int P) {
  return ((size_t)H * D * 6 + (size_t)P * 4 + 15) / 16 * 16 * 2 * kRopeTokensPerCta;
}

static std::pair<const float*, int64_t> rope_angles(const c10::optional<torch::Tensor>& angles, int N, int P,
                                                     const char* who) {
  if (!angles.has_value() || P == 0) return {nullptr, 0};
  TORCH_CHECK(angles->scalar_type() == at::kFloat && angles->is_contiguous() && angles->dim() == 3 &&
                  angles->size(1) == N && angles->size(2) == P,
              who, ": angles must be contiguous fp32 (B or 1, N, P)");
  return {angles->data_ptr<float>(), angles->size(0) == 1 ? 0 : (int64_t)N * P};
}

// qkv (B, N, 3, H, D) -> rotated q and k in qk (B, N, 2, H, D).
void rope_qk_fwd(torch::Tensor qkv, torch::Tensor angles, torch::Tensor pairs, torch::Tensor qk) {
  TORCH_CHECK(qkv.is_contiguous() && qkv.dim() == 5 && qkv.size(2) == 3, "rope_qk_fwd: (B, N, 3, H, D) input");
  TORCH_CHECK(qk.is_contiguous() && qk.size(2) == 2, "rope_qk_fwd: (B, N, 2, H, D) output");
  const int B = (int)qkv.size(0), N = (int)qkv.size(1), H = (int)qkv.size(3), D = (int)qkv.size(4);
  const int P = (int)pairs.size(0);
  TORCH_CHECK(D % 8 == 0 && D <= 256 && P > 0 && P <= D / 2, "rope_qk_fwd: head_dim a multiple of 8 (<= 256), 1..D/2 pairs");
  auto [ang, bstride] = rope_angles(angles, N, P, "rope_qk_fwd");
  TORCH_CHECK(ang != nullptr, "rope_qk_fwd: angles required");
  c10::cuda::CUDAGuard guard(qkv.device());
  const int BN = B * N;
  if (BN == 0) return;
  const size_t smem = rope_fwd_smem(H, D, P);
  C10_CUDA_CHECK(cudaFuncSetAttribute(rope_qk_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rope_qk_fwd_kernel<<<(BN + kRopeTokensPerCta - 1) / kRopeTokensPerCta, 64 * kRopeTokensPerCta, smem,
                       at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(qkv.data_ptr()), ang, pairs.data_ptr<int>(), P, bstride,
      reinterpret_cast<bf16*>(qk.data_ptr()), BN, N, H, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void check_view(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 4 && t.stride(3) == 1 && t.scalar_type() == at::kBFloat16, "attention: ", name,
              " must be a bf16 (B, N, H, D) view with contiguous rows");
  TORCH_CHECK(t.stride(1) % 8 == 0 && t.stride(2) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "attention: ", name, " rows must be 16-byte aligned");
}

// Attention on strided (B, N, H, D) views (e.g. slices of the packed projection); o (B, N, H, D)
// contiguous, lse (B, H, N).
void attention_fwd_strided(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse,
                           double scale) {
  check_view(q, "q");
  check_view(k, "k");
  check_view(v, "v");
  TORCH_CHECK(o.is_contiguous() && lse.is_contiguous(), "attention_fwd_strided: contiguous o and lse");
  const int B = (int)q.size(0), Nq = (int)q.size(1), H = (int)q.size(2), D = (int)q.size(3);
  const int Nk = (int)k.size(1);
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (Nq == 0) return;
  if (attention_fwd_tc(q, k, v, bnhd_strides(q), bnhd_strides(k), bnhd_strides(v), B, H, Nq, Nk, D, o, lse,
                       (float)scale * kLog2e))
    return;
  DISPATCH_HEAD_DIM(D, [&] {
    constexpr int S = HD + 8;
    const size_t smem = (size_t)(kAttnBlockM + 4 * kAttnBlockN) * S * 2;
    auto kern = attn_fwd_kernel<HD>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((Nq + kAttnBlockM - 1) / kAttnBlockM, B * H);
    kern<<<grid, kAttnThreads, smem, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
        reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), H,
        Nq, Nk, (float)scale * kLog2e, bnhd_strides(q), bnhd_strides(k), bnhd_strides(v));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  });
}

// Backward of attention_fwd_strided (+ RoPE when P > 0) into the packed gradient
// dqkv (B, N, 3, H, D): dv and dk are written by the attention backward straight into their slots,
// dq accumulates in fp32 and is cast (and un-rotated, with dk) by rope_qk_bwd_kernel.
void rope_attention_bwd_packed(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                               torch::Tensor lse, c10::optional<torch::Tensor> angles, torch::Tensor pairs,
                               torch::Tensor dqkv, c10::optional<torch::Tensor> dangles, double scale) {
  check_view(q, "q");
  check_view(k, "k");
  check_view(v, "v");
  TORCH_CHECK(dqkv.is_contiguous() && dqkv.dim() == 5 && dqkv.size(2) == 3, "rope_attention_bwd_packed: (B, N, 3, H, D) dqkv");
  TORCH_CHECK(dout.is_contiguous() && o.is_contiguous(), "rope_attention_bwd_packed: contiguous o / do");
  const int B = (int)q.size(0), N = (int)q.size(1), H = (int)q.size(2), D = (int)q.size(3);
  TORCH_CHECK(k.size(1) == N, "rope_attention_bwd_packed: self-attention (Nq == Nk) expected");
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto dq_acc = torch::empty({B, N, H, D}, q.options().dtype(at::kFloat));  // cleared by the delta kernel
  auto dk_view = dqkv.select(2, 1);
  auto dv_view = dqkv.select(2, 2);
  auto delta = torch::empty({B, H, N}, q.options().dtype(at::kFloat));
  DISPATCH_HEAD_DIM(D, [&] {
    const int rows = B * H * N;
    attn_delta_kernel<HD><<<(rows + 255) / 256, 256, 0, stream>>>(
        reinterpret_cast<const bf16*>(o.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
        delta.data_ptr<float>(), H, N, rows, dq_acc.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    if (attention_bwd_tc(q, k, v, dout, bnhd_strides(q), bnhd_strides(k), bnhd_strides(v), bnhd_contiguous(N, H, D),
                         lse, delta, dq_acc, bnhd_strides(dq_acc), dk_view, bnhd_strides(dk_view), dv_view,
                         bnhd_strides(dv_view), B, H, N, N, D, (float)scale))
      return;
    constexpr int S = HD + 8;
    const size_t smem = (size_t)(2 * kAttnBlockN + 2 * kAttnBlockM) * S * 2 + (size_t)kAttnBlockN * (kAttnBlockM + 8) * 2 +
                        2 * kAttnBlockM * 4;
    auto kern = attn_bwd_kernel<HD>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((N + kAttnBlockN - 1) / kAttnBlockN, B * H);
    kern<<<grid, kAttnThreads, smem, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
        reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
        lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
        reinterpret_cast<bf16*>(dk_view.data_ptr()), reinterpret_cast<bf16*>(dv_view.data_ptr()), H, N, N,
        (float)scale, (float)scale * kLog2e, bnhd_strides(q), bnhd_strides(k), bnhd_strides(v),
        bnhd_strides(dq_acc), bnhd_strides(dk_view), bnhd_strides(dv_view));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  });
  const int P = (int)pairs.size(0);
  auto [ang, bstride] = rope_angles(angles, N, P, "rope_attention_bwd_packed");
  const int Pk = ang != nullptr ? P : 0;
  float* dang = (dangles.has_value() && ang != nullptr) ? dangles->data_ptr<float>() : nullptr;
  if (dang != nullptr)
    TORCH_CHECK(dangles->is_contiguous() && dangles->numel() == (int64_t)B * N * P, "rope_attention_bwd_packed: dangles (B, N, P)");
  // y: the rotated q / k the attention read (token stride of the q view's token axis)
  const bf16* y = reinterpret_cast<const bf16*>(q.data_ptr());
  const int64_t y_token_stride = q.stride(1);
  TORCH_CHECK(Pk == 0 || k.data_ptr() == static_cast<const void*>(reinterpret_cast<const bf16*>(q.data_ptr()) + H * D),
              "rope_attention_bwd_packed: k must follow q in the rotated buffer");
  const int BN = B * N;
  if (BN == 0) return;
  const size_t smem = rope_bwd_smem(H, D, Pk);
  C10_CUDA_CHECK(cudaFuncSetAttribute(rope_qk_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rope_qk_bwd_kernel<<<(BN + kRopeTokensPerCta - 1) / kRopeTokensPerCta, 64 * kRopeTokensPerCta, smem, stream>>>(
      dq_acc.data_ptr<float>(), y, y_token_stride, ang, pairs.data_ptr<int>(), Pk, bstride,
      reinterpret_cast<bf16*>(dqkv.data_ptr()), dang, BN, N, H, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mia

// ------------------------------------------------------------------ allocation-free entry point
// See attention_noalloc.h for the contract. The scratch lives in a fixed device array: an fp32
// dQ accumulator followed by the per-row delta = rowsum(dO * O).
#include <cstdio>
#include <mutex>

#include "attention_noalloc.h"

// The scratch array: file scope, internal linkage, one instance per GPU that loads the library.
static __device__ __align__(256) float g_attn_noalloc_scratch[MIA_ATTN_NOALLOC_SCRATCH_FLOATS];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_lock;
float* g_noalloc_scratch_ptr[kNoAllocMaxDevices] = {nullptr};

// Resolves the device address of the scratch array for the current device (first call only).
float* noalloc_scratch_for_current_device(int* device_out) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kNoAllocMaxDevices) return nullptr;
  *device_out = device;
  std::lock_guard<std::mutex> guard(g_noalloc_lock);
  if (g_noalloc_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_attn_noalloc_scratch);
    if (rc != cudaSuccess || ptr == nullptr) {
      std::fprintf(stderr, "mia_attention_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", device,
                   cudaGetErrorString(rc));
      return nullptr;
    }
    g_noalloc_scratch_ptr[device] = static_cast<float*>(ptr);
  }
  return g_noalloc_scratch_ptr[device];
}

template <int D>
int noalloc_launch(const mia::bf16* q, const mia::bf16* k, const mia::bf16* v, const mia::bf16* o,
                   const mia::bf16* dout, const float* lse, mia::bf16* dq, mia::bf16* dk, mia::bf16* dv, int B, int H,
                   int Nq, int Nk, float scale, float* scratch, cudaStream_t stream) {
  using namespace mia;
  const size_t dq_elems = (size_t)B * H * Nq * D;
  float* dq_acc = scratch;
  float* delta = scratch + dq_elems;
  if (cudaMemsetAsync(dq_acc, 0, dq_elems * sizeof(float), stream) != cudaSuccess) return MIA_NOALLOC_ERR_CUDA;
  const int rows = B * H * Nq;
  attn_delta_kernel<D><<<(rows + 255) / 256, 256, 0, stream>>>(o, dout, delta, H, Nq, rows);
  if (cudaGetLastError() != cudaSuccess) return MIA_NOALLOC_ERR_CUDA;
  constexpr int S = D + 8;
  const size_t smem = (size_t)(2 * kAttnBlockN + 2 * kAttnBlockM) * S * 2 + (size_t)kAttnBlockN * (kAttnBlockM + 8) * 2 +
                      2 * kAttnBlockM * 4;
  if (cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MIA_NOALLOC_ERR_CUDA;
  dim3 grid((Nk + kAttnBlockN - 1) / kAttnBlockN, B * H);
  const Strides3 sq{(int64_t)H * Nq * D, (int64_t)Nq * D, D}, sk{(int64_t)H * Nk * D, (int64_t)Nk * D, D};
  attn_bwd_kernel<D><<<grid, kAttnThreads, smem, stream>>>(q, k, v, dout, lse, delta, dq_acc, dk, dv, H, Nq, Nk, scale,
                                                          scale * kLog2e, sq, sk, sk, sq, sk, sk);
  if (cudaGetLastError() != cudaSuccess) return MIA_NOALLOC_ERR_CUDA;
  f32_to_bf16_kernel<<<(unsigned)((dq_elems / 2 + 255) / 256 + 1), 256, 0, stream>>>(dq_acc, dq, dq_elems);
  return cudaGetLastError() == cudaSuccess ? MIA_NOALLOC_OK : MIA_NOALLOC_ERR_CUDA;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int mia_attention_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse, void* dq, void* dk,
    void* dv, int batch, int heads, int seq_q, int seq_k, int head_dim, float scale, void* stream) {
  if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_k <= 0) {
    std::fprintf(stderr, "mia_attention_bwd_noalloc: sizes must be positive\n");
    return MIA_NOALLOC_ERR_ARGS;
  }
  if (head_dim != 32 && head_dim != 64 && head_dim != 128) {
    std::fprintf(stderr, "mia_attention_bwd_noalloc: head_dim must be 32, 64 or 128, got %d\n", head_dim);
    return MIA_NOALLOC_ERR_ARGS;
  }
  const unsigned long long need = (unsigned long long)batch * heads * seq_q * (head_dim + 1);
  if (need > (unsigned long long)MIA_ATTN_NOALLOC_SCRATCH_FLOATS) {
    std::fprintf(stderr,
                 "mia_attention_bwd_noalloc: batch*heads*seq_q*(head_dim+1) = %llu floats of scratch exceeds the "
                 "fixed maximum of %d floats; split the batch or use the allocating entry point\n",
                 need, MIA_ATTN_NOALLOC_SCRATCH_FLOATS);
    return MIA_NOALLOC_ERR_TOO_LARGE;
  }
  const void* tensors[8] = {q, k, v, o, dout, dq, dk, dv};
  for (const void* t : tensors) {
    if (t == nullptr || (reinterpret_cast<uintptr_t>(t) & 15) != 0) {
      std::fprintf(stderr, "mia_attention_bwd_noalloc: q, k, v, o, dout, dq, dk and dv must be non-null and "
                           "16-byte aligned\n");
      return MIA_NOALLOC_ERR_ARGS;
    }
  }
  if (lse == nullptr || (reinterpret_cast<uintptr_t>(lse) & 3) != 0) {
    std::fprintf(stderr, "mia_attention_bwd_noalloc: lse must be non-null and 4-byte aligned\n");
    return MIA_NOALLOC_ERR_ARGS;
  }
  // An error left by earlier work belongs to its owner: report it without consuming it.
  if (cudaPeekAtLastError() != cudaSuccess) {
    std::fprintf(stderr, "mia_attention_bwd_noalloc: a CUDA error is already pending; nothing launched\n");
    return MIA_NOALLOC_ERR_CUDA;
  }
  int device = -1;
  float* scratch = noalloc_scratch_for_current_device(&device);
  if (scratch == nullptr) return MIA_NOALLOC_ERR_CUDA;
  using mia::bf16;
  auto s = static_cast<cudaStream_t>(stream);
  auto cq = static_cast<const bf16*>(q);
  auto ck = static_cast<const bf16*>(k);
  auto cv = static_cast<const bf16*>(v);
  auto co = static_cast<const bf16*>(o);
  auto cd = static_cast<const bf16*>(dout);
  auto oq = static_cast<bf16*>(dq);
  auto ok = static_cast<bf16*>(dk);
  auto ov = static_cast<bf16*>(dv);
  if (head_dim == 32) return noalloc_launch<32>(cq, ck, cv, co, cd, lse, oq, ok, ov, batch, heads, seq_q, seq_k, scale, scratch, s);
  if (head_dim == 64) return noalloc_launch<64>(cq, ck, cv, co, cd, lse, oq, ok, ov, batch, heads, seq_q, seq_k, scale, scratch, s);
  return noalloc_launch<128>(cq, ck, cv, co, cd, lse, oq, ok, ov, batch, heads, seq_q, seq_k, scale, scratch, s);
}
