"""`muvit_mae`: masked autoencoding across scale levels (reference `src/algorithms/muvit_mae.py:37-354`).

Per sample, level weights are drawn from a Dirichlet(alpha) and the kept tokens are sampled by an
exponential race (`log(u) / w`, largest keys win), so some samples keep mostly fine tokens and
others mostly coarse ones. The visible tokens are encoded jointly; one decoder per level
(`decoders.{level}`) reconstructs that level's patches from its mask-token grid, cross-attending in
its first layer to all visible tokens (with their world-coordinate RoPE). The loss is the norm-pix
MSE averaged per level over its hidden patches, then over levels that had any.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from ..data.base import BaseDataset
from ..layers.common.attention import CrossAttention, SelfAttention
from ..layers.common.lora import apply_linear
from ..layers.common.rope import AxialRotaryEmbedding
from ..models.muvit import SPATIAL_RANK
from ..ops.mlp import mlp
from ..ops.norm import layer_norm
from .base import BaseAlgorithm
from .registry import AlgorithmRegistry


def _ln(module: nn.LayerNorm, x: torch.Tensor) -> torch.Tensor:
    return layer_norm(x, module.weight, module.bias, module.eps)


class MuViTDecoderLayer(nn.Module):
    def __init__(self, dim: int, num_heads: int, mlp_ratio: float = 4.0, attention_backend: str = "auto",
                 rotary_base: float = 10000.0, with_cross_attention: bool = False) -> None:
        super().__init__()
        self.rotary = AxialRotaryEmbedding(dim // num_heads, SPATIAL_RANK, base=rotary_base)
        self.norm1 = nn.LayerNorm(dim)
        self.attn = SelfAttention(dim, num_heads, backend=attention_backend)
        if with_cross_attention:
            self.norm_query = nn.LayerNorm(dim)
            self.norm_context = nn.LayerNorm(dim)
            self.cross_attn: CrossAttention | None = CrossAttention(dim, num_heads, backend=attention_backend)
        else:
            self.cross_attn = None
        self.norm2 = nn.LayerNorm(dim)
        self.mlp = nn.Sequential(nn.Linear(dim, int(dim * mlp_ratio)), nn.GELU(), nn.Linear(int(dim * mlp_ratio), dim))

    def forward(self, x, coords, context=None, context_coords=None) -> torch.Tensor:
        rope = self.rotary(coords)
        x = self.attn(_ln(self.norm1, x), rope=rope, residual=x)
        if self.cross_attn is not None:
            if context is None or context_coords is None:
                raise ValueError(
                    "this decoder layer has cross-attention, so it needs both `context` and `context_coords`"
                )
            x = self.cross_attn(
                _ln(self.norm_query, x), _ln(self.norm_context, context), rope=rope,
                context_rope=self.rotary(context_coords), residual=x,
            )
        fc1, fc2 = self.mlp[0], self.mlp[2]
        return mlp(_ln(self.norm2, x), fc1.weight, fc1.bias, fc2.weight, fc2.bias, residual=x)


class MuViTLevelDecoder(nn.Module):
    def __init__(self, dim, num_heads, depth, mlp_ratio, patch_volume, attention_backend="auto",
                 rotary_base=10000.0) -> None:
        super().__init__()
        self.layers = nn.ModuleList(
            MuViTDecoderLayer(dim, num_heads, mlp_ratio, attention_backend, rotary_base, with_cross_attention=(i == 0))
            for i in range(depth)
        )
        self.norm = nn.LayerNorm(dim)
        self.head = nn.Linear(dim, patch_volume)

    def forward(self, x, coords, context, context_coords) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x, coords, context=context, context_coords=context_coords)
        return apply_linear(self.head, _ln(self.norm, x))


@AlgorithmRegistry.register("muvit_mae")
class MuViTMAE(BaseAlgorithm):
    def __init__(
        self,
        model: nn.Module,
        dataset: BaseDataset | None = None,
        input_axes: str | None = None,
        input_key: str = "img",
        bbox_key: str = "bbox",
        mask_ratio: float = 0.75,
        dirichlet_alpha: float = 0.5,
        decoder_embed_dim: int = 384,
        decoder_depth: int = 2,
        decoder_num_heads: int = 6,
        decoder_mlp_ratio: float = 4.0,
        norm_pix_loss: bool = True,
    ) -> None:
        super().__init__(model, dataset)
        if not 0.0 < mask_ratio < 1.0:
            raise ValueError(f"mask_ratio must be in (0, 1), got {mask_ratio}")
        if dirichlet_alpha <= 0.0:
            raise ValueError(f"dirichlet_alpha must be positive, got {dirichlet_alpha}")
        if decoder_depth < 1:
            raise ValueError(f"decoder_depth must be at least 1, got {decoder_depth}")
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        self.input_key = input_key
        self.bbox_key = bbox_key
        self.mask_ratio = mask_ratio
        self.dirichlet_alpha = dirichlet_alpha
        self.norm_pix_loss = norm_pix_loss
        self.encoder = model
        levels = model.num_levels
        self.to_decoder = nn.Linear(model.embed_dim, decoder_embed_dim)
        self.mask_tokens = nn.Parameter(torch.zeros(levels, 1, decoder_embed_dim))
        self.decoders = nn.ModuleList(
            MuViTLevelDecoder(decoder_embed_dim, decoder_num_heads, decoder_depth, decoder_mlp_ratio,
                              model.patch_volume, model.attention_backend)
            for _ in range(levels)
        )
        nn.init.trunc_normal_(self.mask_tokens, std=0.02)

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return tuple(self.decoders)

    def dirichlet_masking(self, batch_size: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        levels, per_level, total = self.encoder.num_levels, self.encoder.patches_per_level, self.encoder.num_patches
        keep = max(1, int(round(total * (1.0 - self.mask_ratio))))
        weights = torch.distributions.Dirichlet(torch.full((levels,), self.dirichlet_alpha, device=device)).sample(
            (batch_size,)
        )
        weights = weights.clamp_min(torch.finfo(weights.dtype).tiny).repeat_interleave(per_level, dim=1)
        u = torch.rand(batch_size, total, device=device)
        keys = u.clamp_min(torch.finfo(u.dtype).tiny).log() / weights
        keep_idx = keys.argsort(dim=1, descending=True)[:, :keep]
        mask = torch.ones(batch_size, total, device=device)
        mask.scatter_(1, keep_idx, 0.0)
        return keep_idx, mask

    def _decode(self, latent, coords, keep_idx, visible_coords) -> torch.Tensor:
        b = latent.shape[0]
        per_level = self.encoder.patches_per_level
        context = apply_linear(self.to_decoder, latent)
        width = context.shape[-1]
        background = torch.cat(
            [self.mask_tokens[i].expand(b, per_level, width) for i in range(self.encoder.num_levels)], dim=1
        ).to(context.dtype)
        tokens = background.scatter(1, keep_idx.unsqueeze(-1).expand(-1, -1, width), context)
        preds = []
        for i, dec in enumerate(self.decoders):
            span = slice(i * per_level, (i + 1) * per_level)
            preds.append(dec(tokens[:, span], coords[:, span], context, visible_coords))
        return torch.cat(preds, dim=1)

    def _loss(self, batch: Any) -> dict[str, torch.Tensor]:
        if self.bbox_key not in batch:
            raise KeyError(
                f"MuViTMAE needs world coordinates under batch[{self.bbox_key!r}], but the batch has only "
                f"{sorted(batch)}"
            )
        volumes = self.encoder.prepare_input(batch[self.input_key], self.input_axes)
        tokens, coords = self.encoder.embed(volumes, batch[self.bbox_key])
        keep_idx, mask = self.dirichlet_masking(tokens.shape[0], tokens.device)
        visible = torch.gather(tokens, 1, keep_idx.unsqueeze(-1).expand(-1, -1, tokens.shape[-1]))
        visible_coords = torch.gather(coords, 1, keep_idx.unsqueeze(-1).expand(-1, -1, SPATIAL_RANK))
        latent = self.encoder.encode(visible, visible_coords)
        prediction = self._decode(latent, coords, keep_idx, visible_coords)
        target = self.encoder.patchify(volumes)
        if self.norm_pix_loss:
            mean = target.mean(dim=-1, keepdim=True)
            var = target.var(dim=-1, keepdim=True)
            target = (target - mean) / torch.sqrt(var + 1e-6)
        per_patch = (prediction.float() - target.float()).pow(2).mean(dim=-1)
        levels, per_level = self.encoder.num_levels, self.encoder.patches_per_level
        m = mask.reshape(-1, levels, per_level)
        hidden = m.sum(dim=-1)
        level_loss = (per_patch.reshape(-1, levels, per_level) * m).sum(dim=-1) / hidden.clamp_min(1.0)
        used = (hidden > 0).to(level_loss.dtype)
        loss = (level_loss * used).sum() / used.sum().clamp_min(1.0)
        return {
            "loss": loss,
            "masked_fraction": mask.mean().detach(),
            "finest_visible_share": (1.0 - m[:, 0].mean(dim=-1)).mean().detach(),
        }

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._loss(batch)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._loss(batch)
