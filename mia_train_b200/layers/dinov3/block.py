"""DINOv3 transformer block (reference `src/layers/dinov3/block.py:27-244`).

Pre-norm `x + ls1(attn(norm1(x)))`, `x + ls2(mlp(norm2(x)))`, over one tensor or a list of crops.
Module names match the reference (`norm1`, `attn`, `ls1`, `norm2`, `mlp`, `ls2`).

Without stochastic depth (the default, `drop_path = 0`), crops are concatenated for every GEMM and
norm, attention runs per crop, and LayerScale plus the residual add are fused into the epilogues of
the output projection and the last MLP layer. With `drop_path > 0` in training, the reference's
sample-subset scheme is kept: a random subset of `max(int(b (1 - p)), 1)` samples runs each branch
and is added back with `index_add(alpha = b / subset)`.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.nn as nn

from ...ops.norm import layer_norm, rms_norm
from ..common.batched_tokens import cat_keep_shapes, uncat_with_shapes
from ..common.layer_scale import LayerScale
from ..common.rms_norm import RMSNorm
from .attention import SelfAttention
from .ffn import Mlp, SwiGLUFFN
from .rope import RopeTables


def _norm(module: nn.Module, x: torch.Tensor) -> torch.Tensor:
    if isinstance(module, nn.LayerNorm) and module.elementwise_affine:
        return layer_norm(x, module.weight, module.bias, module.eps)
    if isinstance(module, RMSNorm):
        return rms_norm(x, module.weight, module.eps)
    return module(x)


class SelfAttentionBlock(nn.Module):
    def __init__(
        self,
        dim: int,
        num_heads: int,
        ffn_ratio: float = 4.0,
        qkv_bias: bool = False,
        proj_bias: bool = True,
        ffn_bias: bool = True,
        drop: float = 0.0,
        attn_drop: float = 0.0,
        init_values=None,
        drop_path: float = 0.0,
        act_layer: Callable[..., nn.Module] = nn.GELU,
        norm_layer: Callable[..., nn.Module] = nn.LayerNorm,
        attn_class: Callable[..., SelfAttention] = SelfAttention,
        ffn_layer: Callable[..., Mlp | SwiGLUFFN] = Mlp,
        mask_k_bias: bool = False,
        use_fa4: bool = False,
        device=None,
    ) -> None:
        super().__init__()
        self.norm1 = norm_layer(dim)
        self.attn: SelfAttention = attn_class(
            dim, num_heads=num_heads, qkv_bias=qkv_bias, proj_bias=proj_bias, attn_drop=attn_drop,
            proj_drop=drop, mask_k_bias=mask_k_bias, use_fa4=use_fa4, device=device,
        )
        self.ls1: nn.Module = LayerScale(dim, init_values=init_values, device=device) if init_values else nn.Identity()
        self.norm2 = norm_layer(dim)
        self.mlp = ffn_layer(
            in_features=dim, hidden_features=int(dim * ffn_ratio), act_layer=act_layer, drop=drop, bias=ffn_bias,
            device=device,
        )
        self.ls2: nn.Module = LayerScale(dim, init_values=init_values, device=device) if init_values else nn.Identity()
        self.sample_drop_ratio = drop_path

    @staticmethod
    def _maybe_index_rope(rope, indices):
        if rope is None or isinstance(rope, RopeTables):
            return rope  # per-token angles shared by every sample: nothing to select
        sin, cos = rope
        if sin.ndim == 4:
            return sin[indices], cos[indices]
        return rope

    @staticmethod
    def _gamma(ls: nn.Module) -> torch.Tensor | None:
        return ls.gamma if isinstance(ls, LayerScale) else None

    def _fused_list(self, x_list: list[torch.Tensor], rope_list) -> list[torch.Tensor]:
        flat, shapes, counts = cat_keep_shapes(x_list)
        h = uncat_with_shapes(_norm(self.norm1, flat), shapes, counts)
        x_attn = self.attn.forward_list(h, rope_list=rope_list, residual_list=x_list, gamma=self._gamma(self.ls1))
        flat, shapes, counts = cat_keep_shapes(x_attn)
        y = self.mlp.forward(_norm(self.norm2, flat), residual=flat, gamma=self._gamma(self.ls2))
        return uncat_with_shapes(y, shapes, counts)

    def _dropped_list(self, x_list: list[torch.Tensor], rope_list) -> list[torch.Tensor]:
        sizes = [x.shape[0] for x in x_list]
        subsets = [max(int(b * (1 - self.sample_drop_ratio)), 1) for b in sizes]
        scales = [b / s for b, s in zip(sizes, subsets, strict=True)]
        idx1 = [torch.randperm(b, device=x.device)[:s] for x, b, s in zip(x_list, sizes, subsets, strict=True)]
        sub1 = [x[i] for x, i in zip(x_list, idx1, strict=True)]
        ropes = [self._maybe_index_rope(r, i) for r, i in zip(rope_list, idx1, strict=True)] if rope_list else rope_list
        flat, shapes, counts = cat_keep_shapes(sub1)
        res1 = self.attn.forward_list(uncat_with_shapes(_norm(self.norm1, flat), shapes, counts), rope_list=ropes)
        x_attn = [
            torch.index_add(x, 0, index=i, source=self.ls1(r).to(x.dtype), alpha=a)
            for x, r, i, a in zip(x_list, res1, idx1, scales, strict=True)
        ]
        idx2 = [torch.randperm(b, device=x.device)[:s] for x, b, s in zip(x_list, sizes, subsets, strict=True)]
        sub2 = [x[i] for x, i in zip(x_attn, idx2, strict=True)]
        flat, shapes, counts = cat_keep_shapes(sub2)
        res2 = self.mlp.forward_list(uncat_with_shapes(_norm(self.norm2, flat), shapes, counts))
        return [
            torch.index_add(x, 0, index=i, source=self.ls2(r).to(x.dtype), alpha=a)
            for x, r, i, a in zip(x_attn, res2, idx2, scales, strict=True)
        ]

    def _forward_list(self, x_list: list[torch.Tensor], rope_list=None) -> list[torch.Tensor]:
        if rope_list is None:
            rope_list = [None] * len(x_list)
        if self.training and self.sample_drop_ratio > 0.0:
            return self._dropped_list(x_list, rope_list)
        return self._fused_list(x_list, rope_list)

    def _forward_with_attention(self, x: torch.Tensor, attention: Callable) -> torch.Tensor:
        """The block on one tensor with a caller-provided attention core `attention(attn, qkv) -> out`."""
        if self.training and self.sample_drop_ratio > 0:
            raise NotImplementedError("blocks with a custom attention core do not support drop_path > 0")
        h = _norm(self.norm1, x)
        out = attention(self.attn, self.attn._qkv(h))
        from ..common.lora import apply_linear

        x_attn = apply_linear(self.attn.proj, out, residual=x, gamma=self._gamma(self.ls1))
        return self.mlp.forward(_norm(self.norm2, x_attn), residual=x_attn, gamma=self._gamma(self.ls2))

    def forward(self, x_or_x_list, rope_or_rope_list=None, *, attention: Callable | None = None, sp=None,
                tokens: tuple[int, int] | None = None):
        """`attention(attn, qkv) -> out` replaces the global attention core (windowed blocks); with `sp`
        (a `parallel.sequence_parallel.SequenceParallel`) the input is this rank's token rows of a
        (B, T) token matrix, `tokens = (B, T)`, and the block runs sequence-parallel."""
        if sp is not None:
            from ...parallel.sequence_parallel import block_forward

            if self.training and self.sample_drop_ratio > 0:
                raise NotImplementedError("sequence-parallel blocks do not support drop_path > 0")
            rope = rope_or_rope_list
            core = attention or (lambda attn, qkv: attn.compute_attention(qkv, rope=rope))
            b, t = tokens
            return block_forward(self, x_or_x_list, sp, lambda qkv: core(self.attn, qkv), b, t)
        if attention is not None:
            return self._forward_with_attention(x_or_x_list, attention)
        if isinstance(x_or_x_list, torch.Tensor):
            return self._forward_list([x_or_x_list], rope_list=[rope_or_rope_list])[0]
        if isinstance(x_or_x_list, list):
            ropes = rope_or_rope_list if rope_or_rope_list is not None else [None] * len(x_or_x_list)
            return self._forward_list(x_or_x_list, rope_list=ropes)
        raise TypeError("SelfAttentionBlock expects a tensor or a list of tensors")
