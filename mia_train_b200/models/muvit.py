"""`muvit3d`: multi-resolution ViT over several scale levels at once (reference `src/models/muvit.py:47-393`).

Each level has its own patch projection (`patch_proj.{level}` = Linear + LayerNorm) and a learned
`level_embed`; all levels' tokens attend jointly in `TransformerBlock`s whose axial RoPE runs on
*world* coordinates: each sample carries a bounding box per level (low and high corner), patch
centres are placed by linear interpolation inside it, and the finest level's box centre is the
origin. Levels must be distinct and ordered finest first (the projections are indexed by position).
The patch projection of a level is a per-patch GEMM on the native kernel followed by the native
LayerNorm.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..layers.common.blocks import TransformerBlock
from ..ops.linear import compute_dtype, linear
from ..ops.norm import layer_norm
from ..ops.patch import patchify_reference
from .base import BaseModel
from .registry import ModelRegistry

SPATIAL_RANK = 3


@ModelRegistry.register("muvit3d")
class MuViT3D(BaseModel):
    def __init__(
        self,
        levels: tuple[int, ...] = (1, 4, 16),
        img_size: tuple[int, int, int] = (64, 64, 64),
        patch_size: tuple[int, int, int] = (8, 8, 8),
        in_channels: int = 1,
        embed_dim: int = 512,
        depth: int = 12,
        num_heads: int = 8,
        mlp_ratio: float = 2.0,
        attention_backend: str = "auto",
        rotary_base: float = 10000.0,
    ) -> None:
        super().__init__()
        levels = tuple(levels)
        img_size = tuple(img_size)  # type: ignore[assignment]
        patch_size = tuple(patch_size)  # type: ignore[assignment]
        if not levels:
            raise ValueError("levels must name at least one scale level")
        if len(set(levels)) != len(levels):
            raise ValueError(f"levels must be distinct, got {levels}")
        if any(lv <= 0 for lv in levels):
            raise ValueError(f"levels must be positive downsampling factors, got {levels}")
        if list(levels) != sorted(levels):
            raise ValueError(
                f"levels must be ordered finest first, got {levels}: the per-level projections are "
                "indexed positionally, so another order would pair a level's data with another's weights"
            )
        if len(img_size) != SPATIAL_RANK or len(patch_size) != SPATIAL_RANK:
            raise ValueError(f"img_size and patch_size must be {SPATIAL_RANK}D, got {img_size} {patch_size}")
        for s, p in zip(img_size, patch_size, strict=True):
            if s % p != 0:
                raise ValueError(f"img_size {img_size} must be divisible by patch_size {patch_size} on every axis")
        self.levels = levels
        self.img_size = img_size
        self.patch_size = patch_size
        self.in_channels = in_channels
        self.embed_dim = embed_dim
        self.mlp_ratio = mlp_ratio
        self.attention_backend = attention_backend
        self.grid_size = tuple(s // p for s, p in zip(img_size, patch_size, strict=True))
        self.patch_proj = nn.ModuleList(
            nn.Sequential(nn.Linear(self.patch_volume, embed_dim), nn.LayerNorm(embed_dim)) for _ in levels
        )
        self.level_embed = nn.Parameter(torch.zeros(len(levels), 1, embed_dim))
        nn.init.trunc_normal_(self.level_embed, std=0.02)
        self.blocks = nn.ModuleList(
            TransformerBlock(embed_dim, num_heads, mlp_ratio, attention_backend, spatial_rank=SPATIAL_RANK,
                             rotary_base=rotary_base)
            for _ in range(depth)
        )
        self.norm = nn.LayerNorm(embed_dim)

    @property
    def num_levels(self) -> int:
        return len(self.levels)

    @property
    def patches_per_level(self) -> int:
        return int(math.prod(self.grid_size))

    @property
    def num_patches(self) -> int:
        return self.patches_per_level * self.num_levels

    @property
    def patch_volume(self) -> int:
        return int(math.prod(self.patch_size)) * self.in_channels

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return tuple(self.blocks)

    def prepare_input(self, batch: torch.Tensor, axes: str) -> torch.Tensor:
        """(B, *axes) -> (B, L, C, D, H, W): the level axis is consumed, one entry per configured level."""
        if "l" not in axes:
            raise ValueError(f"axis order must contain 'l' (scale level), got {axes!r}")
        rest = axes.replace("l", "", 1)
        if not (len(rest) == 3 or (len(rest) == 4 and rest[0] == "c")):
            raise ValueError(f"axis order {axes!r} is not usable by a 3D encoder, got {rest!r} after 'l'")
        if batch.dim() != len(axes) + 1:
            raise ValueError(f"axis order {axes!r} implies a {len(axes) + 1}-D batch, got {tuple(batch.shape)}")
        level_dim = axes.index("l") + 1
        if batch.shape[level_dim] != self.num_levels:
            raise ValueError(
                f"{type(self).__name__} is configured for {self.num_levels} scale levels {self.levels}, but this "
                f"batch carries {batch.shape[level_dim]} on axis 'l' (shape {tuple(batch.shape)})"
            )
        volumes = batch.movedim(level_dim, 1)
        return volumes.unsqueeze(2) if volumes.dim() == 5 else volumes

    def default_bbox(self, batch_size: int, device: torch.device) -> torch.Tensor:
        """Concentric boxes: level l spans level * (size / 2 - 0.5) voxels either side of 0."""
        half = torch.tensor(
            [[lv * (s / 2 - 0.5) for s in self.img_size] for lv in self.levels], dtype=torch.float32, device=device
        )
        return torch.stack((-half, half), dim=1).unsqueeze(0).expand(batch_size, -1, -1, -1)

    def world_coords(self, bbox: torch.Tensor) -> torch.Tensor:
        """(B, L, 2, 3) boxes -> (B, L * patches, 3) patch coordinates, origin at the finest box's centre."""
        b = bbox.shape[0]
        if bbox.shape[1:] != (self.num_levels, 2, SPATIAL_RANK):
            raise ValueError(
                f"bbox must have shape (B, {self.num_levels}, 2, {SPATIAL_RANK}), got {tuple(bbox.shape)}"
            )
        bbox = bbox.to(torch.float32)
        origin = ((bbox[:, 0, 0, :] + bbox[:, 0, 1, :]) / 2).reshape(b, 1, 1, SPATIAL_RANK)
        bbox = bbox - origin
        fracs = [torch.linspace(0.0, 1.0, c, device=bbox.device, dtype=torch.float32) for c in self.grid_size]
        grid = torch.stack(torch.meshgrid(*fracs, indexing="ij"), dim=-1).reshape(1, 1, -1, SPATIAL_RANK)
        low = bbox[:, :, 0, :].unsqueeze(2)
        high = bbox[:, :, 1, :].unsqueeze(2)
        return (low + grid * (high - low)).reshape(b, -1, SPATIAL_RANK)

    def patchify(self, volumes: torch.Tensor) -> torch.Tensor:
        """(B, L, C, D, H, W) -> (B, L * patches, patch_volume), level-major."""
        b, levels = volumes.shape[:2]
        flat = volumes.reshape(b * levels, *volumes.shape[2:])
        rows = patchify_reference(flat, self.patch_size)
        return rows.reshape(b, levels * self.patches_per_level, self.patch_volume)

    def embed(self, volumes: torch.Tensor, bbox: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        expected = (self.num_levels, self.in_channels, *self.img_size)
        if tuple(volumes.shape[1:]) != expected:
            raise ValueError(f"expected input (B, {', '.join(map(str, expected))}), got {tuple(volumes.shape)}")
        if bbox is None:
            bbox = self.default_bbox(volumes.shape[0], volumes.device)
        coords = self.world_coords(bbox.to(volumes.device))
        per_level = self.patchify(volumes).reshape(volumes.shape[0], self.num_levels, self.patches_per_level, -1)
        if volumes.is_cuda:
            per_level = per_level.to(compute_dtype(volumes))
        tokens = []
        for i, proj in enumerate(self.patch_proj):
            lin, norm = proj[0], proj[1]
            t = layer_norm(linear(per_level[:, i], lin.weight, lin.bias), norm.weight, norm.bias, norm.eps)
            tokens.append(t + self.level_embed[i].to(t.dtype))
        return torch.cat(tokens, dim=1), coords

    def encode(self, tokens: torch.Tensor, coords: torch.Tensor) -> torch.Tensor:
        if coords.shape[:2] != tokens.shape[:2]:
            raise ValueError(
                f"every token needs a coordinate: got {tokens.shape[1]} tokens but {coords.shape[1]} coordinates"
            )
        for block in self.blocks:
            tokens = block(tokens, coords)
        return layer_norm(tokens, self.norm.weight, self.norm.bias, self.norm.eps)

    def forward(self, x: torch.Tensor, bbox: torch.Tensor | None = None) -> torch.Tensor:
        tokens, coords = self.embed(x, bbox)
        return self.encode(tokens, coords).mean(dim=1)

    def extra_forward_methods(self) -> tuple[str, ...]:
        return ("embed", "encode")

    def lora_target_groups(self) -> dict[str, tuple[nn.Linear, ...]]:
        return {
            "attn_qkv": tuple(b.attn.qkv for b in self.blocks),
            "attn_proj": tuple(b.attn.proj for b in self.blocks),
            "mlp": tuple(layer for b in self.blocks for layer in (b.mlp[0], b.mlp[2])),
        }

    def tensor_parallel_plan(self):
        from ..parallel.tensor_parallel import vit_block_plan

        return vit_block_plan(self.blocks)

    def flops(self, input_shape: tuple[int, ...]) -> int:
        expected = (self.num_levels, self.in_channels, *self.img_size)
        if tuple(input_shape) != expected:
            raise ValueError(
                f"input_shape {tuple(input_shape)} must be the whole per-sample shape (levels, channels, "
                f"*img_size) = {expected}"
            )
        n, d, depth = self.num_patches, self.embed_dim, len(self.blocks)
        hidden = int(d * self.mlp_ratio)
        per_block = 2 * (4 * n * d * d) + 2 * (2 * n * n * d) + 2 * (2 * n * d * hidden)
        return int(2 * n * self.patch_volume * d + depth * per_block)
