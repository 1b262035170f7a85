// Non-causal multi-head attention, forward and backward, plus the RoPE split/merge around it.
//
// Layouts: q, k, v, dq, dk, dv are (B, H, N, D) bf16; the output o and its gradient do are
// (B, N, H, D) so the output projection reads them as (B*N, H*D) without a transpose.
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
// RoPE: `rope_split_fwd` reads the fused projection (B, N, 3, H, D), rotates channel pairs of q
// and k by per-token angles, and writes q, k, v in (B, H, N, D); `rope_split_bwd` un-rotates dq, dk
// back into the packed gradient and reduces d(angle) per token.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

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
__device__ __forceinline__ void load_rows_async(bf16* smem, const bf16* g, int ld, int row0, int rows, int nvalid) {
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
                                                                float scale_log2) {
  constexpr int S = D + 8;  // padded row stride (elements)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  bf16* Qs = reinterpret_cast<bf16*>(smem_raw);
  bf16* Ks = Qs + kAttnBlockM * S;            // [2][64][S]
  bf16* Vs = Ks + 2 * kAttnBlockN * S;        // [2][64][S]
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kAttnBlockM;
  const bf16* qg = q + (size_t)bh * Nq * D;
  const bf16* kg = k + (size_t)bh * Nk * D;
  const bf16* vg = v + (size_t)bh * Nk * D;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, t = lane % 4;

  load_rows_async<D>(Qs, qg, D, q0, kAttnBlockM, Nq);
  load_rows_async<D>(Ks, kg, D, 0, kAttnBlockN, Nk);
  load_rows_async<D>(Vs, vg, D, 0, kAttnBlockN, Nk);
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
      load_rows_async<D>(Ks + (buf ^ 1) * kAttnBlockN * S, kg, D, (j + 1) * kAttnBlockN, kAttnBlockN, Nk);
      load_rows_async<D>(Vs + (buf ^ 1) * kAttnBlockN * S, vg, D, (j + 1) * kAttnBlockN, kAttnBlockN, Nk);
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
      corr[r] = (m_run[r] == -INFINITY) ? 0.f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mr = m_run[e >> 1];
        const float p = (s[nt][e] == -INFINITY) ? 0.f : exp2f(s[nt][e] - mr);
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

// delta[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d]
template <int D>
__global__ void attn_delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout, float* __restrict__ delta,
                                  int H, int N, int rows) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp_global >= rows) return;
  const int b = warp_global / (H * N);
  const int rem = warp_global % (H * N);
  const int h = rem / N, i = rem % N;
  const size_t off = (((size_t)b * N + i) * H + h) * D;
  float s = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const uint32_t a = *reinterpret_cast<const uint32_t*>(o + off + d);
    const uint32_t c = *reinterpret_cast<const uint32_t*>(dout + off + d);
    s += bf16_lo(a) * bf16_lo(c) + bf16_hi(a) * bf16_hi(c);
  }
#pragma unroll
  for (int x = 16; x > 0; x >>= 1) s += __shfl_xor_sync(0xffffffffu, s, x);
  if (lane == 0) delta[((size_t)b * H + h) * N + i] = s;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_bwd_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, const bf16* __restrict__ dout,
    const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dq_acc, bf16* __restrict__ dk,
    bf16* __restrict__ dv, int H, int Nq, int Nk, float scale, float scale_log2) {
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
  const bf16* qg = q + (size_t)bh * Nq * D;
  const bf16* kg = k + (size_t)bh * Nk * D;
  const bf16* vg = v + (size_t)bh * Nk * D;
  const bf16* dog = dout + ((size_t)b * Nq * H + h) * D;  // row stride H*D

  load_rows_async<D>(Ks, kg, D, k0, kAttnBlockN, Nk);
  load_rows_async<D>(Vs, vg, D, k0, kAttnBlockN, Nk);
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
    load_rows_async<D>(Qs, qg, D, q0, kAttnBlockM, Nq);
    load_rows_async<D>(dOs, dog, H * D, q0, kAttnBlockM, Nq);
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
        st[nt][e] = valid ? exp2f(st[nt][e] * scale_log2 - lse_s[qi_local]) : 0.f;
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
      float* dst = dq_acc + ((size_t)bh * Nq + qi) * D;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        atomicAdd(dst + dt * 8 + 2 * t, dq[dt][2 * r] * scale);
        atomicAdd(dst + dt * 8 + 2 * t + 1, dq[dt][2 * r + 1] * scale);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = my_key0 + g + 8 * r;
    if (key >= Nk) continue;
    bf16* dkr = dk + ((size_t)bh * Nk + key) * D;
    bf16* dvr = dv + ((size_t)bh * Nk + key) * D;
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
// One CTA per token (b, n). The token's packed projection (3*H*D bf16) is staged in shared memory
// with 16-byte loads; per-element rotation roles are built once per CTA from the pair list, and
// cos/sin of the token's P angles are computed once and shared by every head of q and k.
struct RopeRoles {
  int16_t partner;  // -1: channel not rotated
  int16_t pair;
  int8_t second;    // 0: first channel of its pair, 1: second
};

__device__ __forceinline__ void rope_build_roles(RopeRoles* roles, const int* __restrict__ pairs, int P, int D,
                                                 float* cs, float* sn, const float* ang) {
  for (int d = threadIdx.x; d < D; d += blockDim.x) roles[d] = RopeRoles{-1, 0, 0};
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int i1 = pairs[2 * p], i2 = pairs[2 * p + 1];
    roles[i1] = RopeRoles{(int16_t)i2, (int16_t)p, 0};
    roles[i2] = RopeRoles{(int16_t)i1, (int16_t)p, 1};
    float a = ang != nullptr ? ang[p] : 0.f;
    sincosf(a, &sn[p], &cs[p]);
  }
  __syncthreads();
}

// qkv (B, N, 3, H, D) -> q, k, v (B, H, N, D); pairs (P, 2) int32; angles (B or 1, N, P) fp32.
__global__ void rope_split_fwd_kernel(const bf16* __restrict__ qkv, const float* __restrict__ angles,
                                      const int* __restrict__ pairs, int P, int angle_bstride, bf16* __restrict__ q,
                                      bf16* __restrict__ k, bf16* __restrict__ v, int N, int H, int D) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int HD = H * D;
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);                          // [3 * HD]
  float* cs = reinterpret_cast<float*>(smem_raw + 3 * HD * 2);           // [P]
  float* sn = cs + P;                                                    // [P]
  RopeRoles* roles = reinterpret_cast<RopeRoles*>(sn + P);               // [D]
  const int token = blockIdx.x;  // b * N + n
  const int b = token / N, n = token % N;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + (size_t)token * 3 * HD);
  for (int c = threadIdx.x; c < 3 * HD / 8; c += blockDim.x) reinterpret_cast<uint4*>(xs)[c] = src[c];
  const float* ang = (angles != nullptr && P > 0) ? angles + (size_t)b * angle_bstride + (size_t)n * P : nullptr;
  rope_build_roles(roles, pairs, P, D, cs, sn, ang);
  const int chunks_per_head = D / 8;
  for (int c = threadIdx.x; c < 3 * HD / 8; c += blockDim.x) {
    const int which = c / (HD / 8);
    const int rem = c % (HD / 8);
    const int h = rem / chunks_per_head;
    const int d0 = (rem % chunks_per_head) * 8;
    const bf16* x = xs + which * HD + h * D;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = d0 + j;
      const float xi = __bfloat162float(x[d]);
      const RopeRoles r = roles[d];
      if (which < 2 && r.partner >= 0 && ang != nullptr) {
        const float xp = __bfloat162float(x[r.partner]);
        o[j] = r.second ? xi * cs[r.pair] + xp * sn[r.pair] : xi * cs[r.pair] - xp * sn[r.pair];
      } else {
        o[j] = xi;
      }
    }
    bf16* dst = (which == 0 ? q : which == 1 ? k : v) + (((size_t)b * H + h) * N + n) * D + d0;
    *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

// Backward: dqkv (B, N, 3, H, D) from dq (fp32), dk, dv (B, H, N, D); dangles (B, N, P): the CTA
// owns its token, so d(theta_p) = sum over heads and over q, k of (g2 * y1 - g1 * y2) is written
// without atomics (y is the rotated value the attention saw, g its gradient).
__global__ void rope_split_bwd_kernel(const float* __restrict__ dq, const bf16* __restrict__ dk,
                                      const bf16* __restrict__ dv, const bf16* __restrict__ qr,
                                      const bf16* __restrict__ kr, const float* __restrict__ angles,
                                      const int* __restrict__ pairs, int P, int angle_bstride, bf16* __restrict__ dqkv,
                                      float* __restrict__ dangles, int N, int H, int D) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int HD = H * D;
  float* gq = reinterpret_cast<float*>(smem_raw);                 // [HD]
  float* gk = gq + HD;                                            // [HD]
  float* yq = gk + HD;                                            // [HD]
  float* yk = yq + HD;                                            // [HD]
  float* cs = yk + HD;                                            // [P]
  float* sn = cs + P;                                             // [P]
  RopeRoles* roles = reinterpret_cast<RopeRoles*>(sn + P);        // [D]
  const int token = blockIdx.x;
  const int b = token / N, n = token % N;
  const float* ang = (angles != nullptr && P > 0) ? angles + (size_t)b * angle_bstride + (size_t)n * P : nullptr;
  for (int c = threadIdx.x; c < HD / 8; c += blockDim.x) {
    const int h = c / (D / 8), d0 = (c % (D / 8)) * 8;
    const size_t off = (((size_t)b * H + h) * N + n) * D + d0;
    const float4 a = *reinterpret_cast<const float4*>(dq + off);
    const float4 a2 = *reinterpret_cast<const float4*>(dq + off + 4);
    float* gqd = gq + h * D + d0;
    gqd[0] = a.x; gqd[1] = a.y; gqd[2] = a.z; gqd[3] = a.w; gqd[4] = a2.x; gqd[5] = a2.y; gqd[6] = a2.z; gqd[7] = a2.w;
    const uint4 ukv = *reinterpret_cast<const uint4*>(dk + off);
    const uint4 uq = *reinterpret_cast<const uint4*>(qr + off);
    const uint4 uk = *reinterpret_cast<const uint4*>(kr + off);
    const uint32_t w1[4] = {ukv.x, ukv.y, ukv.z, ukv.w}, w2[4] = {uq.x, uq.y, uq.z, uq.w}, w3[4] = {uk.x, uk.y, uk.z, uk.w};
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      gk[h * D + d0 + 2 * hh] = bf16_lo(w1[hh]);
      gk[h * D + d0 + 2 * hh + 1] = bf16_hi(w1[hh]);
      yq[h * D + d0 + 2 * hh] = bf16_lo(w2[hh]);
      yq[h * D + d0 + 2 * hh + 1] = bf16_hi(w2[hh]);
      yk[h * D + d0 + 2 * hh] = bf16_lo(w3[hh]);
      yk[h * D + d0 + 2 * hh + 1] = bf16_hi(w3[hh]);
    }
    // dv passes straight through
    *reinterpret_cast<uint4*>(dqkv + (size_t)token * 3 * HD + 2 * HD + h * D + d0) =
        *reinterpret_cast<const uint4*>(dv + off);
  }
  rope_build_roles(roles, pairs, P, D, cs, sn, ang);
  for (int c = threadIdx.x; c < 2 * HD / 8; c += blockDim.x) {
    const int which = c / (HD / 8);
    const int rem = c % (HD / 8);
    const int h = rem / (D / 8), d0 = (rem % (D / 8)) * 8;
    const float* g = (which == 0 ? gq : gk) + h * D;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = d0 + j;
      const RopeRoles r = roles[d];
      if (r.partner >= 0 && ang != nullptr) {
        const float gi = g[d], gp = g[r.partner];
        o[j] = r.second ? gi * cs[r.pair] - gp * sn[r.pair] : gi * cs[r.pair] + gp * sn[r.pair];
      } else {
        o[j] = g[d];
      }
    }
    *reinterpret_cast<uint4*>(dqkv + (size_t)token * 3 * HD + which * HD + h * D + d0) =
        make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
  if (dangles != nullptr && ang != nullptr) {
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
      const int i1 = pairs[2 * p], i2 = pairs[2 * p + 1];
      float acc = 0.f;
      for (int h = 0; h < H; ++h) {
        acc += gq[h * D + i2] * yq[h * D + i1] - gq[h * D + i1] * yq[h * D + i2];
        acc += gk[h * D + i2] * yk[h * D + i1] - gk[h * D + i1] * yk[h * D + i2];
      }
      dangles[(size_t)token * P + p] = acc;
    }
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

void attention_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse, double scale) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "attention_fwd: contiguous bf16 (B, H, N, D) inputs");
  const int B = (int)q.size(0), H = (int)q.size(1), Nq = (int)q.size(2), D = (int)q.size(3);
  const int Nk = (int)k.size(2);
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (Nq == 0) return;
  DISPATCH_HEAD_DIM(D, [&] {
    constexpr int S = HD + 8;
    const size_t smem = (size_t)(kAttnBlockM + 4 * kAttnBlockN) * S * 2;
    auto kern = attn_fwd_kernel<HD>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((Nq + kAttnBlockM - 1) / kAttnBlockM, B * H);
    kern<<<grid, kAttnThreads, smem, stream>>>(
        reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
        reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), H,
        Nq, Nk, (float)scale * kLog2e);
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
    attn_delta_kernel<HD><<<(rows * 32 + 255) / 256, 256, 0, stream>>>(
        reinterpret_cast<const bf16*>(o.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
        delta.data_ptr<float>(), H, Nq, rows);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
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
        (float)scale * kLog2e);
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

void rope_split_fwd(torch::Tensor qkv, c10::optional<torch::Tensor> angles, torch::Tensor pairs, torch::Tensor q,
                    torch::Tensor k, torch::Tensor v) {
  TORCH_CHECK(qkv.is_contiguous() && qkv.dim() == 5 && qkv.size(2) == 3, "rope_split_fwd: (B, N, 3, H, D) input");
  const int B = (int)qkv.size(0), N = (int)qkv.size(1), H = (int)qkv.size(3), D = (int)qkv.size(4);
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int P = (int)pairs.size(0);
  const float* ang = nullptr;
  int bstride = 0;
  if (angles.has_value() && P > 0) {
    TORCH_CHECK(angles->scalar_type() == at::kFloat && angles->is_contiguous() && angles->size(-1) == P &&
                    angles->size(1) == N,
                "rope_split_fwd: angles must be contiguous fp32 (B or 1, N, P)");
    ang = angles->data_ptr<float>();
    bstride = angles->size(0) == 1 ? 0 : N * P;
  }
  TORCH_CHECK(D % 8 == 0 && D <= 256, "rope_split_fwd: head_dim must be a multiple of 8, at most 256");
  if ((long)B * N == 0) return;
  const size_t smem = (size_t)3 * H * D * 2 + 2 * (size_t)P * 4 + (size_t)D * sizeof(RopeRoles) + 16;
  if (smem > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(rope_split_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rope_split_fwd_kernel<<<B * N, 128, smem, stream>>>(
      reinterpret_cast<const bf16*>(qkv.data_ptr()), ang, pairs.data_ptr<int>(), P, bstride,
      reinterpret_cast<bf16*>(q.data_ptr()), reinterpret_cast<bf16*>(k.data_ptr()), reinterpret_cast<bf16*>(v.data_ptr()),
      N, H, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused backward of rope_split + attention: attention backward into an fp32 dq, then the RoPE
// un-rotation into the packed (B, N, 3, H, D) gradient and per-token d(angle).
void rope_attention_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                        torch::Tensor lse, c10::optional<torch::Tensor> angles, torch::Tensor pairs,
                        torch::Tensor dqkv, c10::optional<torch::Tensor> dangles, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  const int B = (int)q.size(0), H = (int)q.size(1), N = (int)q.size(2), D = (int)q.size(3);
  auto dq_acc = torch::empty(q.sizes(), q.options().dtype(at::kFloat));
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  attention_bwd_core(q, k, v, o, dout, lse, dq_acc, dk, dv, scale);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int P = (int)pairs.size(0);
  const float* ang = nullptr;
  int bstride = 0;
  if (angles.has_value() && P > 0) {
    ang = angles->data_ptr<float>();
    bstride = angles->size(0) == 1 ? 0 : N * P;
  }
  float* dang = (dangles.has_value() && ang != nullptr) ? dangles->data_ptr<float>() : nullptr;
  TORCH_CHECK(D % 8 == 0 && D <= 256, "rope_attention_bwd: head_dim must be a multiple of 8, at most 256");
  const size_t smem = (size_t)4 * H * D * 4 + 2 * (size_t)P * 4 + (size_t)D * sizeof(RopeRoles) + 16;
  if (smem > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(rope_split_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rope_split_bwd_kernel<<<B * N, 128, smem, stream>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<const bf16*>(dk.data_ptr()), reinterpret_cast<const bf16*>(dv.data_ptr()),
      reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()), ang,
      pairs.data_ptr<int>(), P, bstride, reinterpret_cast<bf16*>(dqkv.data_ptr()), dang, N, H, D);
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
  attn_delta_kernel<D><<<(rows * 32 + 255) / 256, 256, 0, stream>>>(o, dout, delta, H, Nq, rows);
  constexpr int S = D + 8;
  const size_t smem = (size_t)(2 * kAttnBlockN + 2 * kAttnBlockM) * S * 2 + (size_t)kAttnBlockN * (kAttnBlockM + 8) * 2 +
                      2 * kAttnBlockM * 4;
  if (cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MIA_NOALLOC_ERR_CUDA;
  dim3 grid((Nk + kAttnBlockN - 1) / kAttnBlockN, B * H);
  attn_bwd_kernel<D><<<grid, kAttnThreads, smem, stream>>>(q, k, v, dout, lse, delta, dq_acc, dk, dv, H, Nq, Nk, scale,
                                                          scale * kLog2e);
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
