"""`simmim`: masked image modelling by mask-token substitution (reference `src/algorithms/simmim.py:114-224`).

The encoder (a DINOv3 model with `forward_features(x, masks)`) replaces hidden patches by its
`mask_token` and runs the full grid; a linear `head` predicts each patch's voxels; the loss is the
L1 error on masked patches (optionally against per-patch normalised targets), with the visible
patches' L1 logged. The mask is drawn in units of `mask_granularity` patches per axis. On CUDA the
loss is one native kernel (`ops.mae.masked_l1`) that reads each target patch straight from the
volume and writes the prediction's gradient in the same pass (no patchified target copy).
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..data.base import BaseDataset
from ..layers.common.lora import apply_linear
from .base import BaseAlgorithm
from .registry import AlgorithmRegistry


def patchify(volumes: torch.Tensor, patch_size: tuple[int, ...]) -> torch.Tensor:
    """(B, C, *spatial) -> (B, prod(grid), C * prod(patch)) in row-major grid order."""
    b, c = volumes.shape[:2]
    spatial = volumes.shape[2:]
    rank = len(patch_size)
    if len(spatial) != rank:
        raise ValueError(f"input has {len(spatial)} spatial axes but patch_size has {rank}")
    for e, p in zip(spatial, patch_size, strict=True):
        if e % p != 0:
            raise ValueError(f"input {tuple(spatial)} is not divisible by patch_size {tuple(patch_size)}")
    grid = [e // p for e, p in zip(spatial, patch_size, strict=True)]
    shape: list[int] = [b, c]
    for g, p in zip(grid, patch_size, strict=True):
        shape += [g, p]
    perm = [0] + [2 + 2 * a for a in range(rank)] + [1] + [3 + 2 * a for a in range(rank)]
    return volumes.reshape(shape).permute(perm).reshape(b, math.prod(grid), c * math.prod(patch_size))


def random_mask(
    grid: tuple[int, ...],
    batch: int,
    ratio: float,
    *,
    granularity: int = 1,
    device: torch.device | None = None,
    generator: torch.Generator | None = None,
) -> torch.Tensor:
    """(B, prod(grid)) bool mask hiding round(ratio * units) coarse units of `granularity` patches."""
    if not 0.0 < ratio < 1.0:
        raise ValueError(f"mask ratio must be in (0, 1), got {ratio}")
    if granularity < 1:
        raise ValueError(f"granularity must be at least 1 patch, got {granularity}")
    coarse = tuple(max(1, math.ceil(e / granularity)) for e in grid)
    units = math.prod(coarse)
    hidden = max(1, int(round(units * ratio)))
    order = torch.rand(batch, units, device=device, generator=generator).argsort(dim=1)
    flat = torch.zeros(batch, units, dtype=torch.bool, device=device)
    flat.scatter_(1, order[:, :hidden], True)
    mask = flat.reshape(batch, *coarse)
    for axis in range(len(grid)):
        mask = mask.repeat_interleave(granularity, dim=axis + 1)
    mask = mask[(slice(None), *(slice(0, e) for e in grid))]
    return mask.reshape(batch, math.prod(grid))


@AlgorithmRegistry.register("simmim")
class SimMIM(BaseAlgorithm):
    def __init__(
        self,
        model: nn.Module,
        dataset: BaseDataset | None = None,
        input_axes: str | None = None,
        input_key: str = "img",
        mask_ratio: float = 0.6,
        mask_granularity: int = 2,
        norm_pix_loss: bool = False,
    ) -> None:
        super().__init__(model, dataset)
        if not hasattr(model, "forward_features"):
            raise TypeError(
                f"{type(model).__name__} has no forward_features, so it cannot substitute a mask token for "
                "hidden patches; use a dinov3_vit or dinov3_vit3d encoder"
            )
        if not 0.0 < mask_ratio < 1.0:
            raise ValueError(f"mask_ratio must be in (0, 1), got {mask_ratio}")
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        self.input_key = input_key
        self.mask_ratio = mask_ratio
        self.mask_granularity = mask_granularity
        self.norm_pix_loss = norm_pix_loss
        self.encoder = model
        self.spatial_rank = int(getattr(model, "spatial_rank", 3))
        patch = model.patch_size
        self.patch_size = (patch,) * self.spatial_rank if isinstance(patch, int) else tuple(patch)
        self.in_chans = int(model.in_chans)
        self.head = nn.Linear(int(model.embed_dim), self.in_chans * math.prod(self.patch_size))

    def _step(self, batch: Any) -> dict[str, torch.Tensor]:
        volumes = self.encoder.prepare_input(batch[self.input_key], self.input_axes)
        grid = tuple(e // p for e, p in zip(volumes.shape[2:], self.patch_size, strict=True))
        mask = random_mask(grid, volumes.shape[0], self.mask_ratio, granularity=self.mask_granularity,
                           device=volumes.device)
        out = self.encoder.forward_features(volumes, mask)
        prediction = apply_linear(self.head, out["x_norm_patchtokens"])
        if prediction.is_cuda and len(self.patch_size) == 3:
            from ..ops.mae import masked_l1

            loss, visible = masked_l1(prediction, volumes, mask, self.patch_size, self.norm_pix_loss)
            return {"loss": loss, "masked_fraction": mask.float().mean(), "visible_l1": visible}
        target = patchify(volumes, self.patch_size)
        if self.norm_pix_loss:
            mean = target.mean(dim=-1, keepdim=True)
            var = target.var(dim=-1, keepdim=True)
            target = (target - mean) / torch.sqrt(var + 1e-6)
        per_patch = F.l1_loss(prediction.float(), target.float(), reduction="none").mean(dim=-1)
        loss = (per_patch * mask).sum() / mask.sum().clamp_min(1.0)
        with torch.no_grad():
            visible = (per_patch * ~mask).sum() / (~mask).sum().clamp_min(1.0)
        return {"loss": loss, "masked_fraction": mask.float().mean(), "visible_l1": visible}

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)
