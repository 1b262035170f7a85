"""Multi-head self- and cross-attention (reference `src/layers/common/attention.py:18-255`).

Module and parameter names match the reference (`qkv`, `proj`; `to_q`, `to_kv`, `proj`). The
projections run on the native tcgen05 GEMM and the attention core on the native fused
RoPE+attention kernel whenever the activations are bf16 on a CUDA device; on the CPU it is PyTorch
SDPA. `attention_backend` keeps the reference's values for config compatibility:

* `"auto"` -- the native kernel on CUDA/bf16, PyTorch on the CPU.
* `"sdpa"` -- always PyTorch SDPA (the reference's fallback), e.g. to compare against.
* `"flash4"` -- FlashAttention-4 is not part of this framework; requesting it is an error that
  names the native kernel instead of silently substituting another kernel.

`counting_kernels(module)` routes every layer through PyTorch math while a step's FLOPs are
counted, because `torch.utils.flop_counter` cannot see custom kernels (the reference does the same
for FA4).
"""

from __future__ import annotations

import contextlib
from collections.abc import Iterator
from typing import Any

import torch
import torch.nn as nn

from ...ops._native import reference_math
from ...ops.attention import attention, attention_reference, rope_attention
from ...parallel.tensor_parallel import rope_to_tp
from .lora import apply_linear
from .rope import RotaryTables

BACKENDS = ("auto", "sdpa", "native", "flash4")


def flash4_status() -> tuple[bool, str]:
    return False, "FlashAttention-4 is not used by this framework; the native sm_100a kernel replaces it"


@contextlib.contextmanager
def counting_kernels(module: nn.Module) -> Iterator[None]:
    """Run every op under `module` as PyTorch math for the duration (for FLOP counting)."""
    with reference_math():
        yield


class _AttentionBase(nn.Module):
    def __init__(self, dim: int, num_heads: int, backend: str = "auto") -> None:
        super().__init__()
        if dim % num_heads != 0:
            raise ValueError(f"dim {dim} must be divisible by num_heads {num_heads}")
        if backend not in BACKENDS:
            raise ValueError(f"backend must be one of {BACKENDS}, got {backend!r}")
        if backend == "flash4":
            raise ValueError(f"backend='flash4' was requested but is unusable: {flash4_status()[1]}")
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim**-0.5
        self.backend = backend

    def selected_backend(self, dtype: torch.dtype, on_cuda: bool) -> str:
        if self.backend != "sdpa" and on_cuda and dtype == torch.bfloat16:
            return "native"
        return "sdpa"


class SelfAttention(_AttentionBase):
    def __init__(self, dim: int, num_heads: int, backend: str = "auto", qkv_bias: bool = True) -> None:
        super().__init__(dim, num_heads, backend)
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)

    def forward(
        self, x: torch.Tensor, rope: Any = None, residual: torch.Tensor | None = None
    ) -> torch.Tensor:
        """(B, N, dim) -> (B, N, dim). With `residual`, returns `residual + attn(x)` (fused add)."""
        b, n, _ = x.shape
        qkv = apply_linear(self.qkv, x).reshape(b, n, 3, self.num_heads, self.head_dim)
        if self.backend == "sdpa":
            with reference_math():
                out = self._attend_packed(qkv, rope)
        else:
            out = self._attend_packed(qkv, rope)
        return apply_linear(self.proj, out.reshape(b, n, -1), residual=residual)

    def _attend_packed(self, qkv: torch.Tensor, rope: Any) -> torch.Tensor:
        if rope is None or isinstance(rope, RotaryTables):
            angles = rope_to_tp(rope.angles, self) if rope is not None else None
            pairs = rope.pairs if rope is not None else None
            return rope_attention(qkv, angles, pairs, self.scale)
        q, k, v = qkv.unbind(dim=2)
        return attention(rope(q), rope(k), v, self.scale)


class CrossAttention(_AttentionBase):
    def __init__(self, dim: int, num_heads: int, backend: str = "auto", qkv_bias: bool = True) -> None:
        super().__init__(dim, num_heads, backend)
        self.to_q = nn.Linear(dim, dim, bias=qkv_bias)
        self.to_kv = nn.Linear(dim, 2 * dim, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)

    def forward(
        self,
        x: torch.Tensor,
        context: torch.Tensor,
        rope: Any = None,
        context_rope: Any = None,
        residual: torch.Tensor | None = None,
    ) -> torch.Tensor:
        b, n, _ = x.shape
        m = context.shape[1]
        q = apply_linear(self.to_q, x).reshape(b, n, self.num_heads, self.head_dim)
        kv = apply_linear(self.to_kv, context).reshape(b, m, 2, self.num_heads, self.head_dim)
        k, v = kv.unbind(dim=2)
        if rope is not None:
            q = rope(q)
        if context_rope is not None:
            k = context_rope(k)
        if self.backend == "sdpa":
            out = attention_reference(q, k, v, self.scale)
        else:
            out = attention(q, k, v, self.scale)
        return apply_linear(self.proj, out.reshape(b, n, -1), residual=residual)
