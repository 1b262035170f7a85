"""Name tables and weight init for the DINOv3 models (reference `src/layers/dinov3/config.py:23-70`)."""

from __future__ import annotations

from collections.abc import Callable
from functools import partial

import torch
import torch.nn as nn

from ..common.layer_scale import LayerScale
from ..common.rms_norm import RMSNorm
from .attention import LinearKMaskedBias
from .ffn import Mlp, SwiGLUFFN
from .patch_embed import PatchEmbed, PatchEmbed3D

ffn_layer_dict: dict[str, Callable[..., Mlp | SwiGLUFFN]] = {
    "mlp": Mlp,
    "swiglu": SwiGLUFFN,
    "swiglu32": partial(SwiGLUFFN, align_to=32),
    "swiglu64": partial(SwiGLUFFN, align_to=64),
    "swiglu128": partial(SwiGLUFFN, align_to=128),
}
norm_layer_dict: dict[str, Callable[..., nn.Module]] = {
    "layernorm": partial(nn.LayerNorm, eps=1e-6),
    "layernormbf16": partial(nn.LayerNorm, eps=1e-5),
    "rmsnorm": RMSNorm,
}
dtype_dict: dict[str, torch.dtype] = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def init_weights_vit(module: nn.Module, name: str = "") -> None:
    if isinstance(module, nn.Linear):
        torch.nn.init.trunc_normal_(module.weight, std=0.02)
        if module.bias is not None:
            nn.init.zeros_(module.bias)
    if isinstance(module, LinearKMaskedBias) and module.bias is not None:
        o = module.out_features
        module.bias_mask.fill_(1)
        module.bias_mask[o // 3 : 2 * o // 3].fill_(0)
    if isinstance(module, (nn.LayerNorm, LayerScale, PatchEmbed, PatchEmbed3D, RMSNorm)):
        module.reset_parameters()
