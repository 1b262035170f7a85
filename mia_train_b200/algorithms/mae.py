"""`mae`: masked autoencoding (reference `src/algorithms/mae.py:16-170`).

Random masking by `argsort` of uniform noise, the visible subset encoded with its coordinates, a
decoder (`decoder_embed`, `mask_token`, `decoder_blocks`, `decoder_norm`, `decoder_head`) that
re-inserts mask tokens in grid order, and a norm-pix MSE on the masked patches. Parameter names
match the reference.

B200 path: only the visible patches are embedded (see `ViT3D.embed`), the mask-token re-insertion
is one gather kernel, and the loss reads each target patch straight from the volume inside one
native kernel that also produces d(prediction).
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from ..data.base import BaseDataset
from ..layers.common.blocks import TransformerBlock
from ..ops.linear import linear
from ..ops.mae import norm_pix_mse, restore_with_mask_token
from ..ops.norm import layer_norm
from .base import BaseAlgorithm
from .registry import AlgorithmRegistry

SPATIAL_RANK = 3


@AlgorithmRegistry.register("mae")
class MAE(BaseAlgorithm):
    def __init__(
        self,
        model: nn.Module,
        dataset: BaseDataset | None = None,
        input_axes: str | None = None,
        input_key: str = "img",
        mask_ratio: float = 0.75,
        decoder_embed_dim: int = 192,
        decoder_depth: int = 2,
        decoder_num_heads: int = 6,
        norm_pix_loss: bool = True,
    ) -> None:
        super().__init__(model, dataset)
        if not 0.0 < mask_ratio < 1.0:
            raise ValueError(f"mask_ratio must be in (0, 1), got {mask_ratio}")
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        self.input_key = input_key
        self.mask_ratio = mask_ratio
        self.norm_pix_loss = norm_pix_loss
        self.encoder = model
        self.decoder_embed = nn.Linear(model.embed_dim, decoder_embed_dim)
        self.mask_token = nn.Parameter(torch.zeros(1, 1, decoder_embed_dim))
        self.decoder_blocks = nn.ModuleList(
            TransformerBlock(
                decoder_embed_dim, decoder_num_heads, 4.0, model.attention_backend, spatial_rank=SPATIAL_RANK
            )
            for _ in range(decoder_depth)
        )
        self.decoder_norm = nn.LayerNorm(decoder_embed_dim)
        self.decoder_head = nn.Linear(decoder_embed_dim, model.patch_volume)
        nn.init.trunc_normal_(self.mask_token, std=0.02)

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return tuple(self.decoder_blocks)

    def random_masking(
        self, batch_size: int, num_tokens: int, device: torch.device
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(keep indices (B, K), mask (B, N) with 1 = hidden, restore permutation (B, N))."""
        keep = max(1, int(round(num_tokens * (1.0 - self.mask_ratio))))
        shuffle = torch.argsort(torch.rand(batch_size, num_tokens, device=device), dim=1)
        restore = torch.argsort(shuffle, dim=1)
        keep_idx = shuffle[:, :keep]
        mask = torch.ones(batch_size, num_tokens, device=device)
        mask.scatter_(1, keep_idx, 0.0)
        return keep_idx, mask, restore

    def decode(self, latent: torch.Tensor, restore: torch.Tensor, coords: torch.Tensor) -> torch.Tensor:
        x = linear(latent, self.decoder_embed.weight, self.decoder_embed.bias)
        x = restore_with_mask_token(x, self.mask_token, restore)
        for block in self.decoder_blocks:
            x = block(x, coords)
        x = layer_norm(x, self.decoder_norm.weight, self.decoder_norm.bias, self.decoder_norm.eps)
        return linear(x, self.decoder_head.weight, self.decoder_head.bias)

    def _loss(self, batch: Any) -> dict[str, torch.Tensor]:
        volumes = self.encoder.prepare_input(batch[self.input_key], self.input_axes)
        b = volumes.shape[0]
        n = self.encoder.num_patches
        keep_idx, mask, restore = self.random_masking(b, n, volumes.device)
        visible, visible_coords = self.encoder.embed(volumes, keep_idx)
        latent = self.encoder.encode(visible, visible_coords)
        coords = self.encoder.patch_coords(b, volumes.device)
        prediction = self.decode(latent, restore, coords)
        loss = norm_pix_mse(prediction, volumes, mask, self.encoder.patch_size, self.norm_pix_loss)
        return {"loss": loss, "masked_fraction": mask.mean().detach()}

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._loss(batch)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._loss(batch)
