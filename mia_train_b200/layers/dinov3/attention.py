"""DINOv3 self-attention (reference `src/layers/dinov3/attention.py:32-198`).

Same module names (`qkv`, `proj`), the optional key-masked bias (`LinearKMaskedBias`: the middle
third of the qkv bias -- the keys' -- is multiplied by a `bias_mask` buffer), RoPE applied to the
patch suffix only (class and register tokens keep angle 0), and `forward_list`, which runs the qkv
and output GEMMs once over the concatenated crops and attention per crop.

On CUDA with bf16 activations the projections use the native tcgen05 GEMM (LayerScale and the
residual add fused into the output projection's epilogue when the block passes them) and the
attention core the native fused RoPE+attention kernel; the rotation pairs channels (i, i + D/2),
i.e. `rope_rotate_half`. `use_fa4` is accepted for config compatibility; FlashAttention-4 is not
part of this framework, so requesting it is an error.
"""

from __future__ import annotations

import contextlib
import math
from collections.abc import Iterator
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ...ops._native import reference_math
from ...ops.attention import rope_attention
from ...parallel.tensor_parallel import rope_to_tp
from ..common.attention import flash4_status
from ..common.batched_tokens import cat_keep_shapes, uncat_with_shapes
from ..common.lora import apply_linear
from .rope import RopeTables


@contextlib.contextmanager
def counting_kernels(module: nn.Module) -> Iterator[None]:
    with reference_math():
        yield


def rope_rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([-x2, x1], dim=-1)


def rope_apply(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor) -> torch.Tensor:
    return (x * cos) + (rope_rotate_half(x) * sin)


class LinearKMaskedBias(nn.Linear):
    bias_mask: torch.Tensor

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        assert self.out_features % 3 == 0
        if self.bias is not None:
            self.register_buffer("bias_mask", torch.full_like(self.bias, fill_value=math.nan))

    def masked_bias(self) -> torch.Tensor | None:
        return self.bias * self.bias_mask.to(self.bias.dtype) if self.bias is not None else None

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        return F.linear(input, self.weight, self.masked_bias())


def half_pairs(head_dim: int, device: torch.device) -> torch.Tensor:
    half = head_dim // 2
    idx = torch.arange(half, dtype=torch.int32)
    return torch.stack([idx, idx + half], dim=1).to(device)


class SelfAttention(nn.Module):
    def __init__(
        self,
        dim: int,
        num_heads: int = 8,
        qkv_bias: bool = False,
        proj_bias: bool = True,
        attn_drop: float = 0.0,
        proj_drop: float = 0.0,
        mask_k_bias: bool = False,
        use_fa4: bool = False,
        device=None,
    ) -> None:
        super().__init__()
        if use_fa4:
            raise ValueError(f"use_fa4=True was requested but is unusable: {flash4_status()[1]}")
        self.use_fa4 = False
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim**-0.5
        cls = LinearKMaskedBias if mask_k_bias else nn.Linear
        self.qkv = cls(dim, dim * 3, bias=qkv_bias, device=device)
        self.attn_drop = nn.Dropout(attn_drop)
        self.proj = nn.Linear(dim, dim, bias=proj_bias, device=device)
        self.proj_drop = nn.Dropout(proj_drop)
        self._pairs: torch.Tensor | None = None

    # -- projections ----------------------------------------------------------------------
    def _qkv(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(self.qkv, LinearKMaskedBias) and self.qkv.bias is not None:
            # the masked key bias replaces the layer's bias on every path (LoRA adapter included)
            return apply_linear(self.qkv, x, bias=self.qkv.masked_bias())
        return apply_linear(self.qkv, x)

    def _pairs_on(self, device: torch.device) -> torch.Tensor:
        if self._pairs is None or self._pairs.device != device:
            self._pairs = half_pairs(self.head_dim, device)
        return self._pairs

    # -- attention core ---------------------------------------------------------------------
    def compute_attention(self, qkv: torch.Tensor, attn_bias=None, rope: Any = None) -> torch.Tensor:
        """(B, N, 3C) projections -> (B, N, C); RoPE on the last `hw` tokens when given."""
        assert attn_bias is None
        b, n, _ = qkv.shape
        c = qkv.shape[-1] // 3
        qkv = qkv.reshape(b, n, 3, self.num_heads, c // self.num_heads)
        angles = None
        if rope is not None:
            if isinstance(rope, RopeTables):
                hw_angles = rope.angles
            else:  # a plain (sin, cos) pair: recover the angle of each channel pair
                sin, cos = rope
                hw_angles = torch.atan2(sin[..., : sin.shape[-1] // 2], cos[..., : cos.shape[-1] // 2])
            prefix = n - hw_angles.shape[-2]
            assert prefix >= 0
            angles = F.pad(rope_to_tp(hw_angles.float(), self), (0, 0, prefix, 0))
            if angles.dim() == 2:
                angles = angles.unsqueeze(0)
        pairs = self._pairs_on(qkv.device) if angles is not None else None
        out = rope_attention(qkv, angles, pairs, self.scale)
        return out.reshape(b, n, c)

    def forward(self, x: torch.Tensor, attn_bias=None, rope=None, residual=None, gamma=None) -> torch.Tensor:
        out = self.compute_attention(self._qkv(x), attn_bias=attn_bias, rope=rope)
        return apply_linear(self.proj, out, residual=residual, gamma=gamma)

    def forward_list(self, x_list, attn_bias=None, rope_list=None, residual_list=None, gamma=None) -> list[torch.Tensor]:
        assert len(x_list) == len(rope_list)
        flat, shapes, counts = cat_keep_shapes(x_list)
        qkv_list = uncat_with_shapes(self._qkv(flat), shapes, counts)
        outs = [self.compute_attention(q, attn_bias=attn_bias, rope=r) for q, r in zip(qkv_list, rope_list, strict=True)]
        flat, shapes, counts = cat_keep_shapes(outs)
        res = None
        if residual_list is not None:
            res, _, _ = cat_keep_shapes(residual_list)
        return uncat_with_shapes(apply_linear(self.proj, flat, residual=res, gamma=gamma), shapes, counts)
