"""DINOv3 patch embeddings, 2D and 3D (reference `src/layers/dinov3/patch_embed.py:43-168`).

A convolution with kernel == stride (`proj`, fan-in uniform init), evaluated as a per-patch GEMM
on the native kernel: the volume (or image) is gathered into patch rows in the convolution's
weight order and multiplied by the flattened kernel.
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch
import torch.nn as nn

from ...ops.linear import compute_dtype, linear
from ...ops.patch import patchify


def make_2tuple(x) -> tuple[int, int]:
    if isinstance(x, (tuple, list)):
        assert len(x) == 2
        return tuple(x)  # type: ignore[return-value]
    assert isinstance(x, int)
    return (x, x)


def make_3tuple(x) -> tuple[int, int, int]:
    if isinstance(x, (tuple, list)):
        assert len(x) == 3, "Input tuple must have length 3"
        return tuple(x)  # type: ignore[return-value]
    assert isinstance(x, int), "Input must be an integer or a tuple of 3 integers"
    return (x, x, x)


class PatchEmbed(nn.Module):
    def __init__(
        self,
        img_size=224,
        patch_size=16,
        in_chans: int = 3,
        embed_dim: int = 768,
        norm_layer: Callable[..., nn.Module] | None = None,
        flatten_embedding: bool = True,
    ) -> None:
        super().__init__()
        hw = make_2tuple(img_size)
        p = make_2tuple(patch_size)
        self.img_size = hw
        self.patch_size = p
        self.patches_resolution = (hw[0] // p[0], hw[1] // p[1])
        self.num_patches = self.patches_resolution[0] * self.patches_resolution[1]
        self.in_chans = in_chans
        self.embed_dim = embed_dim
        self.flatten_embedding = flatten_embedding
        self.proj = nn.Conv2d(in_chans, embed_dim, kernel_size=p, stride=p)
        self.norm = norm_layer(embed_dim) if norm_layer else nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, c, h, w = x.shape
        ph, pw = self.patch_size
        rows = patchify(x.unsqueeze(2), (1, ph, pw), out_dtype=compute_dtype(x) if x.is_cuda else x.dtype)
        out = self.norm(linear(rows, self.proj.weight, self.proj.bias))
        if not self.flatten_embedding:
            out = out.reshape(-1, h // ph, w // pw, self.embed_dim)
        return out

    def reset_parameters(self) -> None:
        k = 1 / (self.in_chans * (self.patch_size[0] ** 2))
        nn.init.uniform_(self.proj.weight, -math.sqrt(k), math.sqrt(k))
        if self.proj.bias is not None:
            nn.init.uniform_(self.proj.bias, -math.sqrt(k), math.sqrt(k))


class PatchEmbed3D(nn.Module):
    def __init__(
        self,
        img_size=(512, 512, 512),
        patch_size=(16, 16, 16),
        in_chans: int = 1,
        embed_dim: int = 768,
        norm_layer: Callable[..., nn.Module] | None = None,
        flatten_embedding: bool = True,
    ) -> None:
        super().__init__()
        dhw = make_3tuple(img_size)
        p = make_3tuple(patch_size)
        self.img_size = dhw
        self.patch_size = p
        self.patches_resolution = tuple(s // q for s, q in zip(dhw, p, strict=True))
        self.num_patches = math.prod(self.patches_resolution)
        self.in_chans = in_chans
        self.embed_dim = embed_dim
        self.flatten_embedding = flatten_embedding
        self.proj = nn.Conv3d(in_chans, embed_dim, kernel_size=p, stride=p)
        self.norm = norm_layer(embed_dim) if norm_layer else nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _, _, d, h, w = x.shape
        pd, ph, pw = self.patch_size
        assert d % pd == 0, f"Input volume depth {d} is not a multiple of patch depth {pd}"
        assert h % ph == 0, f"Input volume height {h} is not a multiple of patch height {ph}"
        assert w % pw == 0, f"Input volume width {w} is not a multiple of patch width {pw}"
        rows = patchify(x, self.patch_size, out_dtype=compute_dtype(x) if x.is_cuda else x.dtype)
        out = self.norm(linear(rows, self.proj.weight, self.proj.bias))
        if not self.flatten_embedding:
            out = out.reshape(-1, d // pd, h // ph, w // pw, self.embed_dim)
        return out

    def reset_parameters(self) -> None:
        k = 1 / (self.in_chans * (self.patch_size[0] ** 3))
        nn.init.uniform_(self.proj.weight, -math.sqrt(k), math.sqrt(k))
        if self.proj.bias is not None:
            nn.init.uniform_(self.proj.bias, -math.sqrt(k), math.sqrt(k))
