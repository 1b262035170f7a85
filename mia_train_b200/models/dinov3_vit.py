"""`dinov3_vit`: the 2D DINOv3 vision transformer (reference `src/models/dinov3_vit.py:44-487`).

The same architecture as `dinov3_vit3d` over images: a Conv2d `PatchEmbed` and the 2D
`RopePositionEmbedding`, with identical parameter names, so Meta's released checkpoints load and
can be inflated into the 3D model through `[init].inflate_2d_to_3d`.
"""

from __future__ import annotations

from typing import Any, Literal

import torch
import torch.nn as nn

from ..layers.dinov3.patch_embed import PatchEmbed
from ..layers.dinov3.rope import RopePositionEmbedding
from .dinov3_vit3d import DinoVisionTransformer3D
from .registry import ModelRegistry


@ModelRegistry.register("dinov3_vit")
class DinoVisionTransformer(DinoVisionTransformer3D):
    spatial_rank = 2

    def __init__(
        self,
        *,
        img_size: int = 224,
        patch_size: int = 16,
        in_chans: int = 3,
        pos_embed_rope_base: float | None = 100.0,
        pos_embed_rope_min_period: float | None = None,
        pos_embed_rope_max_period: float | None = None,
        pos_embed_rope_normalize_coords: Literal["min", "max", "separate"] = "separate",
        pos_embed_rope_shift_coords: float | None = None,
        pos_embed_rope_jitter_coords: float | None = None,
        pos_embed_rope_rescale_coords: float | None = None,
        pos_embed_rope_dtype: str = "bf16",
        embed_dim: int = 768,
        depth: int = 12,
        num_heads: int = 12,
        ffn_ratio: float = 4.0,
        qkv_bias: bool = True,
        drop_path_rate: float = 0.0,
        layerscale_init: float | None = None,
        norm_layer: str = "layernorm",
        ffn_layer: str = "mlp",
        ffn_bias: bool = True,
        proj_bias: bool = True,
        n_storage_tokens: int = 0,
        mask_k_bias: bool = False,
        use_fa4: bool = False,
        untie_cls_and_patch_norms: bool = False,
        untie_global_and_local_cls_norm: bool = False,
        device: Any | None = None,
    ) -> None:
        super().__init__(
            img_size=img_size, patch_size=patch_size, in_chans=in_chans, pos_embed_rope_type="vanilla",
            pos_embed_rope_base=pos_embed_rope_base, pos_embed_rope_min_period=pos_embed_rope_min_period,
            pos_embed_rope_max_period=pos_embed_rope_max_period,
            pos_embed_rope_normalize_coords=pos_embed_rope_normalize_coords,
            pos_embed_rope_shift_coords=pos_embed_rope_shift_coords,
            pos_embed_rope_jitter_coords=pos_embed_rope_jitter_coords,
            pos_embed_rope_rescale_coords=pos_embed_rope_rescale_coords, pos_embed_rope_dtype=pos_embed_rope_dtype,
            embed_dim=embed_dim, depth=depth, num_heads=num_heads, ffn_ratio=ffn_ratio, qkv_bias=qkv_bias,
            drop_path_rate=drop_path_rate, layerscale_init=layerscale_init, norm_layer=norm_layer,
            ffn_layer=ffn_layer, ffn_bias=ffn_bias, proj_bias=proj_bias, n_storage_tokens=n_storage_tokens,
            mask_k_bias=mask_k_bias, use_fa4=use_fa4, untie_cls_and_patch_norms=untie_cls_and_patch_norms,
            untie_global_and_local_cls_norm=untie_global_and_local_cls_norm, device=device,
        )

    def _make_patch_embed(self, img_size, patch_size, in_chans, embed_dim) -> nn.Module:
        return PatchEmbed(img_size=img_size, patch_size=patch_size, in_chans=in_chans, embed_dim=embed_dim,
                          flatten_embedding=False)

    def _make_rope(self, rope_type, base, kwargs) -> nn.Module:
        return RopePositionEmbedding(**kwargs)

    def _rope(self, grid):
        h, w = grid
        return self.rope_embed(H=h, W=w)

    def lora_required_trainable(self) -> tuple[str, ...]:
        return ()

    def prepare_input(self, batch: torch.Tensor, axes: str) -> torch.Tensor:
        """(B, *axes) -> (B, C, H, W); one scale level, two spatial axes."""
        if "l" not in axes:
            raise ValueError(f"axis order must contain 'l' (scale level), got {axes!r}")
        rest = axes.replace("l", "", 1)
        if not (len(rest) == 2 or (len(rest) == 3 and rest[0] == "c")):
            raise ValueError(f"axis order {axes!r} is not usable by a 2D encoder, got {rest!r} after 'l'")
        if batch.dim() != len(axes) + 1:
            raise ValueError(f"axis order {axes!r} implies a {len(axes) + 1}-D batch, got {tuple(batch.shape)}")
        level_dim = axes.index("l") + 1
        if batch.shape[level_dim] != 1:
            raise ValueError(f"{type(self).__name__} is single-scale, but the batch carries {batch.shape[level_dim]} levels")
        images = batch.squeeze(level_dim)
        return images.unsqueeze(1) if images.dim() == 3 else images

    def tensor_parallel_plan(self):
        from ..parallel.tensor_parallel import vit_block_plan

        return vit_block_plan(self.blocks, prefix="blocks")
