"""`synthetic_volumes`: seeded procedural 3D volumes, for benchmarks and tests without data access.

The reference has no such dataset (its data needs `miao` or the HuggingFace Hub). Three generators,
each deterministic in `(seed, index)`:

* `"noise"` -- N(0, 1) voxels, Gaussian-blurred with `sigma`, then z-scored.
* `"blobs"` -- blurred Gaussian noise (`sigma`) quantised to uint8, plus a Poisson(`blob_rate`)
  number of bright solid ellipsoids with semi-axes drawn from `blob_radii`, then z-scored.
* `"voronoi"` -- instance labels from a 3D Voronoi partition of `n_seeds` uniform seeds, with a
  1-voxel boundary (label 0) wherever a 6-neighbour belongs to another cell. The image is a
  per-cell mean intensity U(0.3, 0.7), minus 0.4 on boundary voxels, plus N(0, `noise`) noise,
  blurred with `sigma`. With `classes = K >= 2` the labels are semantic instead: each cell draws a
  class in [1, K) (0 stays the boundary) and its mean intensity is set by its class (evenly spaced
  over [0.25, 0.75], N(0, 0.03) jitter per cell), for `semantic_seg`.

Samples are `{"img": (1, 1, X, Y, Z) float32}` with `sample_axes = "lcxyz"`; the voronoi generator
adds `"label": (1, X, Y, Z) int64`.

`levels = [1, 4, 16]` (finest first, each a whole multiple of the previous) makes a scale pyramid
for multi-level encoders (`muvit3d`): `"img"` is (L, 1, X, Y, Z), level l covering `levels[l]`
times the field of view of level 0 at the same voxel shape, and `"bbox"` is (L, 2, 3) float32,
the concentric world-coordinate box of each level (voxels of level 0, centred on a random offset).
The coarsest level is drawn by the generator; each finer level is the central `1 / ratio` crop of
the next coarser one upsampled trilinearly, plus fresh detail from the same generator, so the
levels agree where they overlap. Multi-level sampling takes the noise and blobs generators.
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn.functional as F
import torch.utils.data as data

from .base import BaseDataset
from .registry import DataRegistry

GENERATORS = ("noise", "blobs", "voronoi")


def gaussian_kernel1d(sigma: float) -> torch.Tensor:
    radius = max(1, int(math.ceil(3.0 * sigma)))
    x = torch.arange(-radius, radius + 1, dtype=torch.float32)
    k = torch.exp(-0.5 * (x / sigma) ** 2)
    return k / k.sum()


def gaussian_blur3d(volume: torch.Tensor, sigma: float) -> torch.Tensor:
    """Separable Gaussian blur of a (X, Y, Z) float volume with reflect padding."""
    if sigma <= 0:
        return volume
    k = gaussian_kernel1d(sigma)
    r = (k.numel() - 1) // 2
    x = volume[None, None]
    for axis in range(3):
        shape = [1, 1, 1, 1, 1]
        shape[2 + axis] = k.numel()
        pad = [0, 0, 0, 0, 0, 0]
        pad[2 * (2 - axis)] = r
        pad[2 * (2 - axis) + 1] = r
        x = F.conv3d(F.pad(x, pad, mode="reflect" if volume.shape[axis] > r else "replicate"), k.view(shape))
    return x[0, 0]


def _zscore(v: torch.Tensor) -> torch.Tensor:
    return (v - v.mean()) / v.std().clamp_min(1e-6)


def noise_volume(shape: tuple[int, int, int], sigma: float, gen: torch.Generator) -> torch.Tensor:
    return _zscore(gaussian_blur3d(torch.randn(shape, generator=gen), sigma))


def blobs_volume(
    shape: tuple[int, int, int],
    sigma: float,
    blob_rate: float,
    blob_radii: tuple[float, float],
    gen: torch.Generator,
) -> torch.Tensor:
    base = _zscore(gaussian_blur3d(torch.randn(shape, generator=gen), sigma))
    vol = (base * 32.0 + 96.0).clamp(0, 255)
    count = int(torch.poisson(torch.tensor([blob_rate]), generator=gen).item())
    grids = [torch.arange(s, dtype=torch.float32) for s in shape]
    for _ in range(count):
        centre = [float(torch.rand((), generator=gen)) * s for s in shape]
        radii = [
            blob_radii[0] + float(torch.rand((), generator=gen)) * (blob_radii[1] - blob_radii[0])
            for _ in range(3)
        ]
        lo = [max(0, int(c - r) - 1) for c, r in zip(centre, radii, strict=True)]
        hi = [min(s, int(c + r) + 2) for c, r, s in zip(centre, radii, shape, strict=True)]
        if any(h <= low for low, h in zip(lo, hi, strict=True)):
            continue
        dx = ((grids[0][lo[0]:hi[0]] - centre[0]) / radii[0]) ** 2
        dy = ((grids[1][lo[1]:hi[1]] - centre[1]) / radii[1]) ** 2
        dz = ((grids[2][lo[2]:hi[2]] - centre[2]) / radii[2]) ** 2
        inside = (dx[:, None, None] + dy[None, :, None] + dz[None, None, :]) <= 1.0
        region = vol[lo[0]:hi[0], lo[1]:hi[1], lo[2]:hi[2]]
        region[inside] = 230.0
    vol = vol.round().to(torch.uint8)
    return _zscore(vol.float())


def voronoi_volume(
    shape: tuple[int, int, int], n_seeds: int, noise: float, sigma: float, gen: torch.Generator, classes: int = 0
) -> tuple[torch.Tensor, torch.Tensor]:
    seeds = torch.rand(n_seeds, 3, generator=gen) * torch.tensor(shape, dtype=torch.float32)
    coords = torch.stack(
        torch.meshgrid(*[torch.arange(s, dtype=torch.float32) + 0.5 for s in shape], indexing="ij"),
        dim=-1,
    ).reshape(-1, 3)
    nearest = torch.empty(coords.shape[0], dtype=torch.int64)
    chunk = 1 << 16
    for start in range(0, coords.shape[0], chunk):
        nearest[start:start + chunk] = torch.cdist(coords[start:start + chunk], seeds).argmin(dim=1)
    cells = (nearest + 1).reshape(shape)
    boundary = torch.zeros(shape, dtype=torch.bool)
    for axis in range(3):
        a = cells.narrow(axis, 0, shape[axis] - 1)
        b = cells.narrow(axis, 1, shape[axis] - 1)
        differ = a != b
        boundary.narrow(axis, 1, shape[axis] - 1).logical_or_(differ)
    labels = cells.masked_fill(boundary, 0)
    if classes >= 2:  # semantic labels: each cell draws a class in [1, classes), its mean intensity follows it
        cls = torch.randint(1, classes, (n_seeds + 1,), generator=gen)
        means = 0.25 + 0.5 * (cls.float() - 1) / max(1, classes - 2) + 0.03 * torch.randn(n_seeds + 1, generator=gen)
        labels = cls[cells].masked_fill(boundary, 0)
    else:
        means = 0.3 + 0.4 * torch.rand(n_seeds + 1, generator=gen)
    image = means[cells] - 0.4 * boundary.float()
    image = image + noise * torch.randn(shape, generator=gen)
    return gaussian_blur3d(image, sigma), labels


def _draw(s: dict[str, Any], shape: tuple[int, int, int], gen: torch.Generator) -> torch.Tensor:
    if s["generator"] == "noise":
        return noise_volume(shape, float(s["sigma"]), gen)
    return blobs_volume(shape, float(s["sigma"]), float(s["blob_rate"]), tuple(s["blob_radii"]), gen)


def pyramid(s: dict[str, Any], gen: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
    """(L, X, Y, Z) levels, finest first, and their (L, 2, 3) concentric boxes."""
    shape = tuple(int(v) for v in s["shape"])
    levels = tuple(int(v) for v in s["levels"])
    out = [_draw(s, shape, gen)]  # the coarsest level
    for fine, coarse in zip(reversed(levels[:-1]), reversed(levels[1:]), strict=True):
        ratio = coarse // fine
        crop = [n // ratio for n in shape]
        lo = [(n - c) // 2 for n, c in zip(shape, crop, strict=True)]
        centre = out[-1][lo[0]:lo[0] + crop[0], lo[1]:lo[1] + crop[1], lo[2]:lo[2] + crop[2]]
        up = F.interpolate(centre[None, None], size=shape, mode="trilinear", align_corners=False)[0, 0]
        out.append(_zscore(up + _draw(s, shape, gen)))
    volumes = torch.stack(out[::-1])
    offset = (torch.rand(3, generator=gen) - 0.5) * 2.0 * max(shape)
    half = torch.tensor([[lv * (n / 2 - 0.5) for n in shape] for lv in levels], dtype=torch.float32)
    bbox = torch.stack((offset - half, offset + half), dim=1)
    return volumes, bbox


class _SyntheticSource(data.Dataset):
    def __init__(self, settings: dict[str, Any]) -> None:
        self.s = settings

    def __len__(self) -> int:
        return int(self.s["samples_per_epoch"])

    def __getitem__(self, index: int) -> dict[str, Any]:
        s = self.s
        gen = torch.Generator().manual_seed(int(s["seed"]) * 1_000_003 + int(index))
        shape = tuple(int(v) for v in s["shape"])
        sample: dict[str, Any] = {}
        if len(s["levels"]) > 1:
            volumes, bbox = pyramid(s, gen)
            return {"img": volumes[:, None].contiguous(), "bbox": bbox}
        if s["generator"] == "noise":
            img = noise_volume(shape, float(s["sigma"]), gen)
        elif s["generator"] == "blobs":
            img = blobs_volume(shape, float(s["sigma"]), float(s["blob_rate"]), tuple(s["blob_radii"]), gen)
        else:
            img, labels = voronoi_volume(shape, int(s["n_seeds"]), float(s["noise"]), float(s["sigma"]), gen,
                                         int(s["classes"]))
            sample["label"] = labels[None]
        sample["img"] = img[None, None].contiguous()
        return sample


@DataRegistry.register("synthetic_volumes")
class SyntheticVolumes(BaseDataset):
    def __init__(
        self,
        generator: str = "noise",
        shape: tuple[int, int, int] = (64, 64, 64),
        samples_per_epoch: int = 64,
        seed: int = 0,
        sigma: float = 2.0,
        blob_rate: float = 50.0,
        blob_radii: tuple[float, float] = (2.0, 8.0),
        n_seeds: int = 300,
        noise: float = 0.08,
        levels: tuple[int, ...] = (1,),
        classes: int = 0,
    ) -> None:
        super().__init__()
        self.settings = self.resolve_settings(
            generator=generator,
            shape=shape,
            samples_per_epoch=samples_per_epoch,
            seed=seed,
            sigma=sigma,
            blob_rate=blob_rate,
            blob_radii=blob_radii,
            n_seeds=n_seeds,
            noise=noise,
            levels=levels,
            classes=classes,
        )

    @classmethod
    def resolve_settings(cls, **kwargs: Any) -> dict[str, Any]:
        defaults = {
            "generator": "noise",
            "shape": (64, 64, 64),
            "samples_per_epoch": 64,
            "seed": 0,
            "sigma": 2.0,
            "blob_rate": 50.0,
            "blob_radii": (2.0, 8.0),
            "n_seeds": 300,
            "noise": 0.08,
            "levels": (1,),
            "classes": 0,
        }
        unknown = sorted(set(kwargs) - set(defaults))
        if unknown:
            raise ValueError(f"synthetic_volumes got unknown key(s) {unknown}; valid: {sorted(defaults)}")
        out = {**defaults, **kwargs}
        if out["generator"] not in GENERATORS:
            raise ValueError(f"generator must be one of {GENERATORS}, got {out['generator']!r}")
        out["shape"] = tuple(int(v) for v in out["shape"])
        if len(out["shape"]) != 3 or min(out["shape"]) < 1:
            raise ValueError(f"shape must be three positive extents, got {out['shape']}")
        out["blob_radii"] = tuple(float(v) for v in out["blob_radii"])
        levels = tuple(int(v) for v in out["levels"])
        if not levels or levels[0] < 1 or any(b <= a or b % a for a, b in zip(levels, levels[1:], strict=False)):
            raise ValueError(f"levels must be increasing, each a whole multiple of the previous; got {levels}")
        if len(levels) > 1:
            if out["generator"] == "voronoi":
                raise ValueError("multi-level samples take the noise or blobs generator")
            ratio = max(b // a for a, b in zip(levels, levels[1:], strict=False))
            if any(n % ratio for n in out["shape"]):
                raise ValueError(f"shape {out['shape']} must divide by the level ratio {ratio}")
        out["levels"] = levels
        out["classes"] = int(out["classes"])
        if out["classes"] and (out["classes"] < 2 or out["generator"] != "voronoi"):
            raise ValueError(f"classes = {out['classes']}: semantic classes (>= 2) take the voronoi generator")
        if int(out["samples_per_epoch"]) < 1:
            raise ValueError("samples_per_epoch must be >= 1")
        return out

    @property
    def sample_axes(self) -> str:
        return "lcxyz"

    def build_dataset(self) -> data.Dataset:
        return _SyntheticSource(self.settings)
