"""On-device multi-crop views and iBOT block masks (reference `src/algorithms/dinov3/multicrop.py:50-246`).

* `random_resized_crop`: per sample, a random sub-box (volume fraction from `scale`, per-axis
  aspect jitter, random centre, optional flips and a quarter turn in the first two axes) resampled
  to `out_size` by `affine_grid` + `grid_sample` (linear, reflection padding).
* `photometric`: per-sample brightness/contrast, separable Gaussian blur (grouped convolution) and
  additive noise, each gated by its probability.
* `block_mask`: for the first `sample_probability` fraction of samples, random boxes are added
  until a target fraction (spread linearly over `ratio`) of the grid is masked, up to 64 attempts,
  a box being accepted only if it adds at most the remaining count. The reference runs this on the
  training device with a host synchronisation per attempt; here it runs on the host with NumPy
  and the finished mask is copied once.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class AugmentationConfig:
    brightness: float = 0.4
    contrast: float = 0.4
    intensity_prob: float = 0.8
    blur_prob: float = 0.5
    blur_sigma: tuple[float, float] = (0.1, 2.0)
    noise_std: float = 0.05
    noise_prob: float = 0.5
    flip_prob: float = 0.5
    rotate_prob: float = 0.5


def random_resized_crop(volumes, out_size, scale, *, flip_prob=0.5, rotate_prob=0.5, generator=None):
    b, c = volumes.shape[:2]
    rank = volumes.ndim - 2
    dev = volumes.device

    def draw(*shape):
        return torch.rand(*shape, device=dev, generator=generator)

    fraction = draw(b) * (scale[1] - scale[0]) + scale[0]
    side = fraction.pow(1.0 / rank).unsqueeze(1).expand(b, rank)
    side = (side * torch.exp((draw(b, rank) - 0.5) * 0.4)).clamp(0.05, 1.0)
    centre = (draw(b, rank) * 2 - 1) * (1 - side)
    if flip_prob > 0:
        side = side * torch.where(draw(b, rank) < flip_prob, -1.0, 1.0)
    theta = torch.zeros(b, rank, rank + 1, device=dev, dtype=torch.float32)
    theta[:, :, rank] = centre
    diag = torch.diag_embed(side)
    if rotate_prob > 0 and rank >= 2:
        turn = draw(b) < rotate_prob
        rot = torch.eye(rank, device=dev).expand(b, rank, rank).clone()
        rot[turn, 0, 0] = 0.0
        rot[turn, 1, 1] = 0.0
        rot[turn, 0, 1] = -1.0
        rot[turn, 1, 0] = 1.0
        diag = torch.bmm(rot, diag)
    theta[:, :, :rank] = diag
    grid = F.affine_grid(theta, [b, c, *out_size], align_corners=False)
    return F.grid_sample(volumes.float(), grid, mode="bilinear", padding_mode="reflection", align_corners=False)


def _gaussian_blur(volumes: torch.Tensor, sigma: torch.Tensor) -> torch.Tensor:
    rank = volumes.ndim - 2
    b, c = volumes.shape[:2]
    radius = 4
    offs = torch.arange(-radius, radius + 1, device=volumes.device, dtype=torch.float32)
    kernel = torch.exp(-(offs[None, :] ** 2) / (2 * sigma[:, None] ** 2))
    kernel = kernel / kernel.sum(dim=1, keepdim=True)
    conv = (F.conv1d, F.conv2d, F.conv3d)[rank - 1]
    out = volumes
    for axis in range(rank):
        shape = [b, 1] + [1] * rank
        shape[2 + axis] = 2 * radius + 1
        weight = kernel.reshape(shape).repeat_interleave(c, dim=0)
        merged = out.reshape(1, b * c, *out.shape[2:])
        pad = [0] * (2 * rank)
        pad[2 * (rank - 1 - axis)] = radius
        pad[2 * (rank - 1 - axis) + 1] = radius
        out = conv(F.pad(merged, pad, mode="reflect"), weight, groups=b * c).reshape(b, c, *out.shape[2:])
    return out


def photometric(views: torch.Tensor, config: AugmentationConfig, *, generator=None) -> torch.Tensor:
    b = views.shape[0]
    dev = views.device
    per_sample = (b,) + (1,) * (views.ndim - 1)

    def draw(*shape):
        return torch.rand(*shape, device=dev, generator=generator)

    apply_int = (draw(b) < config.intensity_prob).view(per_sample)
    brightness = 1 + (draw(b).view(per_sample) * 2 - 1) * config.brightness
    contrast = 1 + (draw(b).view(per_sample) * 2 - 1) * config.contrast
    mean = views.mean(dim=tuple(range(1, views.ndim)), keepdim=True)
    views = torch.where(apply_int, (views - mean) * contrast + mean * brightness, views)
    if config.blur_prob > 0:
        lo, hi = config.blur_sigma
        blurred = _gaussian_blur(views, draw(b) * (hi - lo) + lo)
        views = torch.where((draw(b) < config.blur_prob).view(per_sample), blurred, views)
    if config.noise_prob > 0 and config.noise_std > 0:
        noise = torch.randn(views.shape, device=dev, generator=generator) * config.noise_std
        views = torch.where((draw(b) < config.noise_prob).view(per_sample), views + noise, views)
    return views


def block_mask(
    grid: tuple[int, ...],
    batch: int,
    ratio: tuple[float, float],
    *,
    sample_probability: float = 0.5,
    min_patches: int = 4,
    max_aspect: float = 1 / 0.3,
    device: torch.device | None = None,
    generator: torch.Generator | None = None,
) -> torch.Tensor:
    """(batch, prod(grid)) bool masks; RNG draws come from torch's CPU generator (seedable)."""
    total = math.prod(grid)
    rank = len(grid)
    masks = np.zeros((batch, *grid), dtype=bool)
    n_masked = int(batch * sample_probability)
    if n_masked > 0:
        targets = torch.linspace(ratio[0], ratio[1], n_masked).tolist()
        # enough uniform draws for every attempt, taken in one call
        draws = torch.rand(n_masked, 64, 2 + rank, generator=generator).numpy()
        log_aspect = math.log(max_aspect)
        for s in range(n_masked):
            wanted = int(targets[s] * total)
            filled = 0
            view = masks[s]
            for a in range(64):
                if filled >= wanted:
                    break
                remaining = wanted - filled
                span = max(min_patches + 1, remaining)
                area = min_patches + draws[s, a, 0] * (span - min_patches)
                aspect = math.exp((draws[s, a, 1] - 0.5) * 2 * log_aspect)
                side = max(1, int(round((area * aspect) ** (1.0 / rank))))
                ext = [min(side, grid[i]) for i in range(rank)]
                corner = [int(draws[s, a, 2 + i] * (grid[i] - ext[i] + 1)) for i in range(rank)]
                window = tuple(slice(corner[i], corner[i] + ext[i]) for i in range(rank))
                fresh = int((~view[window]).sum())
                if fresh == 0 or fresh > remaining:
                    continue
                view[window] = True
                filled += fresh
    out = torch.from_numpy(masks.reshape(batch, total))
    return out.to(device, non_blocking=True) if device is not None else out
