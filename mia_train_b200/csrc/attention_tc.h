// Host entry points of the tcgen05 attention kernels (attention_tc.cu), used by attention.cu.
#pragma once

#include <torch/extension.h>

#include <cstdint>

namespace mia {

// Element strides of a (B, H, N, D) view whose rows of D are contiguous.
struct Strides3 {
  int64_t b, h, n;
};

// Launches the tcgen05 forward when it supports the problem (head dim 32 or 64, TMA-compatible
// strides and alignment, path enabled) and returns true; returns false without launching
// otherwise. o: (B, Nq, H, D) bf16 contiguous; lse: (B, H, Nq) fp32, log2 domain.
bool attention_fwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, Strides3 qs,
                      Strides3 ks, Strides3 vs, int B, int H, int Nq, int Nk, int D, torch::Tensor& o,
                      torch::Tensor& lse, float scale_log2);

// Backward counterpart (same applicability rules; additionally 16-byte aligned dq_acc / dk / dv
// rows). dq_acc: fp32, zeroed by the caller, receives dQ by atomic adds; dk / dv: bf16 views.
// delta = rowsum(dO * O) (B, H, Nq) fp32; lse from the forward.
bool attention_bwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                      const torch::Tensor& dout, Strides3 qs, Strides3 ks, Strides3 vs, Strides3 dos,
                      const torch::Tensor& lse, const torch::Tensor& delta, torch::Tensor& dq_acc, Strides3 dqs,
                      torch::Tensor& dk, Strides3 dks, torch::Tensor& dv, Strides3 dvs, int B, int H, int Nq, int Nk,
                      int D, float scale);

// 1 (default): use the tcgen05 kernels where they apply; 0: always the warp-level kernels.
void set_tc_attention_mode(int64_t mode);
int64_t tc_attention_mode();
// Number of tcgen05 attention launches so far (host counter, for tests and launch accounting).
int64_t tc_attention_launches();

}  // namespace mia
