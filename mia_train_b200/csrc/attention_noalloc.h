// mia_attention_bwd_noalloc: attention backward for callers that cannot allocate device memory.
//
// This entry point has no counterpart in the reference (mia-train): it is an addition of this
// framework for code that may not call cudaMalloc -- for example a host runtime or plugin that
// owns the device memory budget and only hands out the tensors it manages, or code that runs
// while the caching allocator must not grow. It computes the gradients of the allocating
// `attention_bwd` binding from the forward pass's saved q, k, v, o and lse, but always with the
// warp-level (mma.sync) backward kernels of attention.cu: `attention_bwd` runs the tcgen05 kernels
// for head dims 32 and 64 instead. The two paths agree to bf16 rounding, not bit for bit.
//
// Contract
// * Inputs q, k, v (B, H, N, D) bf16; o and dout (B, N, H, D) bf16; lse (B, H, Nq) fp32, as written
//   by `attention_fwd`. Outputs dq, dk, dv (B, H, N, D) bf16, allocated by the caller. D must be
//   32, 64 or 128. `stream` is a cudaStream_t (nullptr for the legacy default stream).
// * Every tensor pointer must be non-null and 16-byte aligned (the kernels move 16-byte vectors);
//   lse must be non-null and 4-byte aligned. Anything else returns MIA_NOALLOC_ERR_ARGS before a
//   launch. The size check runs first, so an oversized problem is refused whatever its pointers.
// * Scratch memory is a fixed file-scope device array of MIA_ATTN_NOALLOC_SCRATCH_FLOATS floats
//   (8 MiB per GPU, held by every GPU that loads the library until the process exits). A call
//   needs B*H*Nq*(D+1) floats of it; larger problems are rejected with MIA_NOALLOC_ERR_TOO_LARGE
//   and a message on stderr, before anything is launched.
// * Nothing is allocated: no cudaMalloc/cudaFree, no library routine that allocates. The first call
//   on a device resolves the scratch array's device address with cudaGetSymbolAddress (with that
//   device current); make that first call before any stream capture.
// * Every call on a device shares the same scratch array, which keeps the previous call's contents;
//   the call clears the part that must start at zero itself. Calls that overlap on the GPU (on
//   different streams, or from different threads) race on the scratch array: serialise them.
// * Returns MIA_NOALLOC_OK (0) or a negative error code. A CUDA error already pending on entry is
//   left in place (for its owner to see) and the call returns MIA_NOALLOC_ERR_CUDA without
//   launching; each launch is checked as it is issued. Kernel failures surface, as usual for CUDA,
//   at the caller's next synchronisation.
#pragma once

#define MIA_ATTN_NOALLOC_SCRATCH_FLOATS (1 << 21)

#define MIA_NOALLOC_OK 0
#define MIA_NOALLOC_ERR_ARGS (-1)
#define MIA_NOALLOC_ERR_TOO_LARGE (-2)
#define MIA_NOALLOC_ERR_CUDA (-3)

#ifdef __cplusplus
extern "C" {
#endif

int mia_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                              const float* lse, void* dq, void* dk, void* dv, int batch, int heads, int seq_q,
                              int seq_k, int head_dim, float scale, void* stream);

#ifdef __cplusplus
}
#endif
