"""`dinov3_vit3d`: the DINOv3 vision transformer for volumes (reference `src/models/dinov3_vit3d.py:44-587`).

Same constructor keywords, parameter names and outputs as the reference: `patch_embed`
(PatchEmbed3D), `cls_token`, `storage_tokens` (registers), `rope_embed` (vanilla 3D or
superposition), `blocks.N`, `norm` (+ optional untied `cls_norm` / `local_cls_norm`),
`mask_token`; `forward_features(_list)` returning `x_norm_clstoken` / `x_storage_tokens` /
`x_norm_patchtokens` / `x_prenorm` / `masks`, `get_intermediate_layers`, `patch_features`, LoRA
target groups, and the superposition `depth_scale` kept trainable under LoRA.

Differences:
* RoPE tables are computed once per crop and forward and shared by all blocks, unless a
  train-time coordinate augmentation is configured, in which case every block draws its own (as
  the reference does for every block).
* New: `window_size` / `global_every` give windowed attention. Blocks whose index i satisfies
  `(i + 1) % global_every != 0` attend within non-overlapping `window_size^3` token windows of the
  patch grid, with the class and register tokens visible to every window and attending globally;
  every `global_every`-th block attends globally. `window_size = 0` (the default) is the
  reference's all-global model.
* New: `tensor_parallel_plan()` -- colwise qkv / fc1 / w1 / w2 and rowwise proj / fc2 / w3, so
  `[parallelism].tp > 1` works on this model.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from typing import Any, Literal

import torch
import torch.nn as nn

from ..layers.dinov3.block import SelfAttentionBlock, _norm
from ..layers.dinov3.config import dtype_dict, ffn_layer_dict, init_weights_vit, norm_layer_dict
from ..layers.dinov3.ffn import SwiGLUFFN
from ..layers.dinov3.patch_embed import PatchEmbed3D
from ..layers.dinov3.rope import RopePositionEmbedding3D, RopePositionEmbedding3DSuperposition
from ..utils.module_ops import named_apply
from .base import BaseModel
from .registry import ModelRegistry

SPATIAL_RANK = 3
ROPE_TYPES = ("vanilla", "superposition")


def prepare_volume_input(model: nn.Module, batch: torch.Tensor, axes: str) -> torch.Tensor:
    """(B, *axes) -> (B, C, D, H, W) for single-scale 3D encoders."""
    if "l" not in axes:
        raise ValueError(f"axis order must contain 'l' (scale level), got {axes!r}")
    rest = axes.replace("l", "", 1)
    if not (len(rest) == SPATIAL_RANK or (len(rest) == SPATIAL_RANK + 1 and rest[0] == "c")):
        raise ValueError(
            f"axis order {axes!r} is not usable by a 3D encoder: after the level axis it must be three "
            f"spatial axes, optionally preceded by 'c', got {rest!r}"
        )
    if batch.dim() != len(axes) + 1:
        raise ValueError(f"axis order {axes!r} implies a {len(axes) + 1}-D batch, got {tuple(batch.shape)}")
    level_dim = axes.index("l") + 1
    if batch.shape[level_dim] != 1:
        raise ValueError(
            f"{type(model).__name__} is single-scale, but this batch carries {batch.shape[level_dim]} scale "
            f"levels on axis 'l' (shape {tuple(batch.shape)}); configure the dataset for one level"
        )
    volumes = batch.squeeze(level_dim)
    return volumes.unsqueeze(1) if volumes.dim() == SPATIAL_RANK + 1 else volumes


@ModelRegistry.register("dinov3_vit3d")
class DinoVisionTransformer3D(BaseModel):
    def __init__(
        self,
        *,
        img_size: int = 224,
        patch_size: int = 16,
        in_chans: int = 1,
        pos_embed_rope_type: Literal["vanilla", "superposition"] = "vanilla",
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
        window_size: int = 0,
        global_every: int = 0,
        device: Any | None = None,
    ) -> None:
        super().__init__()
        if norm_layer not in norm_layer_dict:
            raise ValueError(f"unknown norm_layer {norm_layer!r}; expected one of {sorted(norm_layer_dict)}")
        if ffn_layer not in ffn_layer_dict:
            raise ValueError(f"unknown ffn_layer {ffn_layer!r}; expected one of {sorted(ffn_layer_dict)}")
        if pos_embed_rope_dtype not in dtype_dict:
            raise ValueError(f"unknown pos_embed_rope_dtype {pos_embed_rope_dtype!r}; expected one of {sorted(dtype_dict)}")
        if pos_embed_rope_type not in ROPE_TYPES:
            raise ValueError(f"unknown pos_embed_rope_type {pos_embed_rope_type!r}; expected one of {list(ROPE_TYPES)}")
        if window_size < 0 or global_every < 0:
            raise ValueError("window_size and global_every must be >= 0")
        norm_cls = norm_layer_dict[norm_layer]
        self.num_features = self.embed_dim = embed_dim
        self.n_blocks = depth
        self.num_heads = num_heads
        self.patch_size = patch_size
        self.in_chans = in_chans
        self.img_size = img_size
        self.window_size = window_size
        self.global_every = global_every
        self.patch_embed = self._make_patch_embed(img_size, patch_size, in_chans, embed_dim)
        self.cls_token = nn.Parameter(torch.empty(1, 1, embed_dim, device=device))
        self.n_storage_tokens = n_storage_tokens
        if n_storage_tokens > 0:
            self.storage_tokens = nn.Parameter(torch.empty(1, n_storage_tokens, embed_dim, device=device))
        rope_kwargs = dict(
            embed_dim=embed_dim, num_heads=num_heads, base=pos_embed_rope_base,
            min_period=pos_embed_rope_min_period, max_period=pos_embed_rope_max_period,
            normalize_coords=pos_embed_rope_normalize_coords, shift_coords=pos_embed_rope_shift_coords,
            jitter_coords=pos_embed_rope_jitter_coords, rescale_coords=pos_embed_rope_rescale_coords,
            dtype=dtype_dict[pos_embed_rope_dtype], device=device,
        )
        self.rope_embed = self._make_rope(pos_embed_rope_type, pos_embed_rope_base, rope_kwargs)
        ffn_cls = ffn_layer_dict[ffn_layer]
        self.blocks = nn.ModuleList(
            SelfAttentionBlock(
                dim=embed_dim, num_heads=num_heads, ffn_ratio=ffn_ratio, qkv_bias=qkv_bias, proj_bias=proj_bias,
                ffn_bias=ffn_bias, drop_path=drop_path_rate, norm_layer=norm_cls, act_layer=nn.GELU,
                ffn_layer=ffn_cls, init_values=layerscale_init, mask_k_bias=mask_k_bias, use_fa4=use_fa4,
                device=device,
            )
            for _ in range(depth)
        )
        self.chunked_blocks = False
        self.norm = norm_cls(embed_dim)
        self.untie_cls_and_patch_norms = untie_cls_and_patch_norms
        self.cls_norm = norm_cls(embed_dim) if untie_cls_and_patch_norms else None
        self.untie_global_and_local_cls_norm = untie_global_and_local_cls_norm
        self.local_cls_norm = norm_cls(embed_dim) if untie_global_and_local_cls_norm else None
        self.head = nn.Identity()
        self.mask_token = nn.Parameter(torch.empty(1, embed_dim, device=device))
        self.init_weights()

    # -- spatial-rank hooks (the 2D model overrides these) -------------------------------------
    spatial_rank = SPATIAL_RANK

    def _make_patch_embed(self, img_size, patch_size, in_chans, embed_dim) -> nn.Module:
        return PatchEmbed3D(img_size=img_size, patch_size=patch_size, in_chans=in_chans, embed_dim=embed_dim,
                            flatten_embedding=False)

    def _make_rope(self, rope_type, base, kwargs) -> nn.Module:
        if rope_type == "vanilla":
            return RopePositionEmbedding3D(**kwargs)
        return RopePositionEmbedding3DSuperposition(depth_base=10.0 * base if base is not None else None, **kwargs)

    def _rope(self, grid: tuple[int, ...]):
        d, h, w = grid
        return self.rope_embed(D=d, H=h, W=w)

    def init_weights(self) -> None:
        self.rope_embed._init_weights()
        nn.init.normal_(self.cls_token, std=0.02)
        if self.n_storage_tokens > 0:
            nn.init.normal_(self.storage_tokens, std=0.02)
        nn.init.zeros_(self.mask_token)
        named_apply(init_weights_vit, self)

    # -- geometry -----------------------------------------------------------------------------
    @property
    def grid_size(self) -> tuple[int, ...]:
        side = self.img_size // self.patch_size
        return (side,) * self.spatial_rank

    @property
    def num_patches(self) -> int:
        return int(math.prod(self.grid_size))

    @property
    def n_prefix(self) -> int:
        return 1 + self.n_storage_tokens

    def is_windowed(self, index: int) -> bool:
        if self.window_size <= 0:
            return False
        return self.global_every <= 0 or (index + 1) % self.global_every != 0

    # -- tokens -------------------------------------------------------------------------------
    def prepare_tokens_with_masks(self, x: torch.Tensor, masks=None) -> tuple[torch.Tensor, tuple[int, int, int]]:
        x = self.patch_embed(x)
        b = x.shape[0]
        grid = tuple(x.shape[1:-1])
        x = x.flatten(1, len(grid))
        if masks is not None:
            x = torch.where(masks.unsqueeze(-1), self.mask_token.to(x.dtype).unsqueeze(0), x)
            cls_token = self.cls_token
        else:
            cls_token = self.cls_token + 0 * self.mask_token
        if self.n_storage_tokens > 0:
            storage = self.storage_tokens
        else:
            storage = torch.empty(1, 0, cls_token.shape[-1], dtype=cls_token.dtype, device=cls_token.device)
        x = torch.cat([cls_token.expand(b, -1, -1).to(x.dtype), storage.expand(b, -1, -1).to(x.dtype), x], dim=1)
        return x, grid

    def _rope_augmented(self) -> bool:
        r = self.rope_embed
        return self.training and any(v is not None for v in (r.shift_coords, r.jitter_coords, r.rescale_coords))

    def _run_blocks(self, tokens_list: list[torch.Tensor], grids: list[tuple[int, int, int]],
                    take: set[int] | None = None) -> tuple[list[torch.Tensor], list[list[torch.Tensor]]]:
        shared = None if self._rope_augmented() else [self._rope(g) for g in grids]
        sp = getattr(self, "_sequence_parallel", None)
        if sp is not None:
            return self._run_blocks_sequence_parallel(sp, tokens_list, grids, shared, take)
        taken: list[list[torch.Tensor]] = []
        for i, blk in enumerate(self.blocks):
            ropes = shared if shared is not None else [self._rope(g) for g in grids]
            if self.is_windowed(i):
                tokens_list = [
                    self._windowed_block(blk, t, g, r) for t, g, r in zip(tokens_list, grids, ropes, strict=True)
                ]
            else:
                tokens_list = blk(tokens_list, ropes)
            if take is not None and i in take:
                taken.append(list(tokens_list))
        return tokens_list, taken

    def _run_blocks_sequence_parallel(self, sp, tokens_list, grids, shared, take):
        """Blocks on this rank's token rows (crop by crop); tokens are gathered again after the last block."""
        from ..layers.dinov3.windowed import windowed_core

        outs: list[torch.Tensor] = []
        taken: list[list[torch.Tensor]] = [[] for _ in self.blocks] if take is not None else []
        for c, (tok, grid) in enumerate(zip(tokens_list, grids, strict=True)):
            b, t, _ = tok.shape
            x_r, _ = sp.split(tok)
            for i, blk in enumerate(self.blocks):
                rope = shared[c] if shared is not None else self._rope(grid)
                core = windowed_core(grid, rope, self.n_prefix, self.window_size) if self.is_windowed(i) else None
                x_r = blk(x_r, rope, attention=core, sp=sp, tokens=(b, t))
                if take is not None and i in take:
                    taken[i].append(sp.gather(x_r, b, t))
            outs.append(sp.gather(x_r, b, t))
        if take is not None:
            taken = [t for i, t in enumerate(taken) if i in take]
        return outs, taken

    def enable_sequence_parallel(self, sp) -> None:
        """Run the blocks sequence-parallel (`parallel.sequence_parallel.SequenceParallel`); call after
        the blocks were sharded by `apply_tensor_parallel`."""
        from ..parallel.sequence_parallel import mark_partial_params

        self._sequence_parallel = sp
        mark_partial_params(list(self.blocks), sp.group)

    def _windowed_block(self, blk: SelfAttentionBlock, x: torch.Tensor, grid, rope) -> torch.Tensor:
        """One block with window attention for patch tokens and global attention for the prefix."""
        from ..layers.dinov3.windowed import windowed_block_forward

        return windowed_block_forward(blk, x, grid, rope, self.n_prefix, self.window_size)

    def forward_features_list(self, x_list: list[torch.Tensor], masks_list: list[torch.Tensor | None]) -> list[dict]:
        tokens_list, grids = [], []
        for t_x, t_masks in zip(x_list, masks_list, strict=True):
            tok, grid = self.prepare_tokens_with_masks(t_x, t_masks)
            tokens_list.append(tok)
            grids.append(grid)
        tokens_list, _ = self._run_blocks(tokens_list, grids)
        out = []
        p = self.n_prefix
        for idx, (x, masks) in enumerate(zip(tokens_list, masks_list, strict=True)):
            if self.untie_cls_and_patch_norms or self.untie_global_and_local_cls_norm:
                if self.untie_global_and_local_cls_norm and self.training and idx == 1:
                    cls_reg = _norm(self.local_cls_norm, x[:, :p])
                if self.untie_cls_and_patch_norms:
                    cls_reg = _norm(self.cls_norm, x[:, :p])
                else:
                    cls_reg = _norm(self.norm, x[:, :p])
                patch = _norm(self.norm, x[:, p:])
            else:
                xn = _norm(self.norm, x)
                cls_reg, patch = xn[:, :p], xn[:, p:]
            out.append({
                "x_norm_clstoken": cls_reg[:, 0],
                "x_storage_tokens": cls_reg[:, 1:],
                "x_norm_patchtokens": patch,
                "x_prenorm": x,
                "masks": masks,
            })
        return out

    def forward_features(self, x, masks=None):
        if isinstance(x, torch.Tensor):
            assert not isinstance(masks, list), "a single input takes a single mask, not a list"
            return self.forward_features_list([x], [masks])[0]
        assert isinstance(masks, list), "a list of crops needs a matching list of masks"
        return self.forward_features_list(x, masks)

    def _get_intermediate_layers_not_chunked(self, x: torch.Tensor, n: int | Sequence[int] = 1) -> list[torch.Tensor]:
        tok, grid = self.prepare_tokens_with_masks(x)
        total = len(self.blocks)
        take = set(range(total - n, total)) if isinstance(n, int) else set(n)
        _, taken = self._run_blocks([tok], [grid], take)
        outputs = [t[0] for t in taken]
        assert len(outputs) == len(take), f"only {len(outputs)} / {len(take)} blocks found"
        return outputs

    def get_intermediate_layers(
        self,
        x: torch.Tensor,
        *,
        n: int | Sequence[int] = 1,
        reshape: bool = False,
        return_class_token: bool = False,
        return_extra_tokens: bool = False,
        norm: bool = True,
    ):
        outputs = self._get_intermediate_layers_not_chunked(x, n)
        p = self.n_prefix
        if norm:
            normed = []
            for o in outputs:
                if self.untie_cls_and_patch_norms:
                    normed.append(torch.cat((_norm(self.cls_norm, o[:, :p]), _norm(self.norm, o[:, p:])), dim=1))
                else:
                    normed.append(_norm(self.norm, o))
            outputs = normed
        cls_tokens = [o[:, 0] for o in outputs]
        extra = [o[:, 1:p] for o in outputs]
        outputs = [o[:, p:] for o in outputs]
        if reshape:
            b = x.shape[0]
            grid = [s // self.patch_size for s in x.shape[-self.spatial_rank:]]
            perm = (0, self.spatial_rank + 1, *range(1, self.spatial_rank + 1))
            outputs = [o.reshape(b, *grid, -1).permute(*perm).contiguous() for o in outputs]
        if not return_class_token and not return_extra_tokens:
            return tuple(outputs)
        if return_class_token and not return_extra_tokens:
            return tuple(zip(outputs, cls_tokens, strict=True))
        if not return_class_token and return_extra_tokens:
            return tuple(zip(outputs, extra, strict=True))
        return tuple(zip(outputs, cls_tokens, extra, strict=True))

    def forward(self, *args, is_training: bool = False, **kwargs):
        ret = self.forward_features(*args, **kwargs)
        if is_training:
            return ret
        assert isinstance(ret, dict), "forward() over a list of crops requires is_training=True"
        return self.head(ret["x_norm_clstoken"])

    def patch_features(self, x: torch.Tensor):
        out = self.forward_features(x)
        grid = tuple(s // self.patch_size for s in x.shape[-self.spatial_rank:])
        return out["x_norm_patchtokens"], grid

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return tuple(self.blocks)

    def lora_target_groups(self) -> dict[str, tuple[nn.Linear, ...]]:
        return {
            "attn_qkv": tuple(b.attn.qkv for b in self.blocks),
            "attn_proj": tuple(b.attn.proj for b in self.blocks),
            "mlp": tuple(m for b in self.blocks for m in b.mlp.modules() if isinstance(m, nn.Linear)),
        }

    def lora_required_trainable(self) -> tuple[str, ...]:
        return ("rope_embed.depth_scale",) if isinstance(self.rope_embed, RopePositionEmbedding3DSuperposition) else ()

    def prepare_input(self, batch: torch.Tensor, axes: str) -> torch.Tensor:
        return prepare_volume_input(self, batch, axes)

    def extra_forward_methods(self) -> tuple[str, ...]:
        return ("forward_features", "get_intermediate_layers")

    def tensor_parallel_plan(self) -> Any:
        from ..parallel.tensor_parallel import vit_block_plan

        return vit_block_plan(self.blocks, prefix="blocks")

    def flops(self, input_shape: tuple[int, ...]) -> int:
        r = self.spatial_rank
        if len(input_shape) < r:
            raise ValueError(f"input_shape {tuple(input_shape)} needs at least {r} axes")
        if len(input_shape) > r and input_shape[-r - 1] != self.in_chans:
            raise ValueError(f"input_shape {tuple(input_shape)}: the channel axis must be in_chans {self.in_chans}")
        spatial = input_shape[-r:]
        if any(e % self.patch_size for e in spatial):
            raise ValueError(f"input_shape {tuple(input_shape)}: spatial axes must be multiples of {self.patch_size}")
        grid = tuple(s // self.patch_size for s in spatial)
        patches = int(math.prod(grid))
        n = patches + self.n_prefix
        d = self.embed_dim
        mlp = self.blocks[0].mlp
        ffn = 2 * (3 * n * d * mlp.w1.out_features) if isinstance(mlp, SwiGLUFFN) else 2 * (2 * n * d * mlp.fc1.out_features)
        total = 2 * patches * self.patch_size**r * self.in_chans * d
        for i in range(len(self.blocks)):
            keys = (self.window_size**3 + self.n_prefix) if self.is_windowed(i) else n
            total += 2 * (4 * n * d * d) + 2 * (2 * n * keys * d) + ffn
        return int(total)
