"""Volumetric EM augmentation run in the dataloader workers, one sample at a time.

Same operations and gating as the reference's `src/data/augment.py:61-377`:

* a random signed permutation of the spatial axes (`rotate = "full"`: all 48 in 3D; `"inplane"`:
  the sectioning axis z stays in its slot and may only flip, 16 in 3D), drawn once per sample and
  applied identically to image and labels;
* section shifts: one spatial axis is drawn, each section along it is selected with probability
  `shift_slice_prob` and rolled in-plane by an integer in `[-shift_magnitude, shift_magnitude]`
  per remaining axis (image and labels together);
* section drops (image only): sections along a random axis are zeroed with `drop_slice_prob`;
* intensity jitter (image only): `x * U(1-mul, 1+mul) + U(-add, add)`;
* additive noise (image only): Gaussian with standard deviation `U(0, 1) * noise_scale`.

Every operation except the rotation is applied with probability 1/2. Geometry runs before the
photometric operations. Labels have no channel axis, so their spatial axes are located from the
layout with `c` removed.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch

SPATIAL_AXES = "xyz"
SECTION_AXIS = "z"
ROTATIONS = ("none", "inplane", "full")
APPLY_PROB = 0.5


def spatial_dims(axes: str) -> tuple[int, ...]:
    """Negative (end-relative) positions of the spatial axes within a per-sample layout string."""
    n = len(axes)
    return tuple(i - n for i, a in enumerate(axes) if a in SPATIAL_AXES)


def _absolute(t: torch.Tensor, dims: Sequence[int]) -> list[int]:
    return [d % t.ndim for d in dims]


def rot90(
    tensors: Sequence[torch.Tensor],
    dims: Sequence[Sequence[int]],
    fixed_slot: int | None = None,
) -> tuple[torch.Tensor, ...]:
    """Apply one random signed axis permutation to every tensor (slot `fixed_slot` is not moved)."""
    rank = len(dims[0])
    movable = [s for s in range(rank) if s != fixed_slot]
    shuffled = [movable[i] for i in torch.randperm(len(movable)).tolist()]
    source_of = list(range(rank))
    for slot, src in zip(movable, shuffled, strict=True):
        source_of[slot] = src
    flip = (torch.rand(rank) < 0.5).tolist()
    results = []
    for t, t_dims in zip(tensors, dims, strict=True):
        ax = _absolute(t, t_dims)
        moved = [s for s in range(rank) if source_of[s] != s]
        extents = {t.shape[ax[s]] for s in moved}
        if len(extents) > 1:
            raise ValueError(
                f"rotation exchanges spatial slots {moved} of a {tuple(t.shape)} tensor whose "
                "extents differ; a permutation must preserve the shape"
            )
        flipped = [ax[s] for s in range(rank) if flip[s]]
        if flipped:
            t = torch.flip(t, dims=flipped)
        order = list(range(t.ndim))
        for slot, a in enumerate(ax):
            order[a] = ax[source_of[slot]]
        results.append(t.permute(order).contiguous())
    return tuple(results)


def shift_sections(
    tensors: Sequence[torch.Tensor],
    dims: Sequence[Sequence[int]],
    prob: float,
    magnitude: int,
) -> tuple[torch.Tensor, ...]:
    rank = len(dims[0])
    slot = int(torch.randint(rank, ()).item())
    length = tensors[0].shape[_absolute(tensors[0], dims[0])[slot]]
    chosen = torch.nonzero(torch.rand(length) < prob).flatten().tolist()
    if not chosen or magnitude == 0:
        return tuple(tensors)
    offsets = {
        i: tuple(int(torch.randint(-magnitude, magnitude + 1, ()).item()) for _ in range(rank - 1))
        for i in chosen
    }
    results = []
    for t, t_dims in zip(tensors, dims, strict=True):
        ax = _absolute(t, t_dims)
        axis = ax[slot]
        plane = tuple(a - (1 if a > axis else 0) for a in ax if a != axis)
        front = t.clone().movedim(axis, 0)
        for i, shift in offsets.items():
            front[i].copy_(torch.roll(front[i], shifts=shift, dims=plane))
        results.append(front.movedim(0, axis))
    return tuple(results)


def drop_sections(image: torch.Tensor, dims: Sequence[int], prob: float) -> torch.Tensor:
    ax = _absolute(image, dims)
    axis = ax[int(torch.randint(len(ax), ()).item())]
    gone = torch.nonzero(torch.rand(image.shape[axis]) < prob).flatten()
    if gone.numel() == 0:
        return image
    return image.clone().index_fill_(axis, gone, 0.0)


def intensity_jitter(image: torch.Tensor, mul: float, add: float) -> torch.Tensor:
    scale = float(torch.empty(()).uniform_(1.0 - mul, 1.0 + mul).item())
    shift = float(torch.empty(()).uniform_(-add, add).item())
    return image * scale + shift


def additive_noise(image: torch.Tensor, scale: float) -> torch.Tensor:
    sigma = float(torch.rand(()).item()) * scale
    return image + torch.randn_like(image) * sigma


class VolumeAugmentation:
    """Callable `sample dict -> sample dict` applying the configured operations."""

    def __init__(
        self,
        rotate: str = "none",
        drop_slice_prob: float = 0.0,
        shift_slice_prob: float = 0.0,
        shift_magnitude: int = 10,
        intensity: bool = False,
        mul_intensity: float = 0.1,
        add_intensity: float = 0.1,
        noise_scale: float = 0.0,
        sample_axes: str | None = None,
        image_keys: tuple[str, ...] = ("img",),
        label_keys: tuple[str, ...] = ("label",),
    ) -> None:
        if rotate not in ROTATIONS:
            raise ValueError(f"rotate must be one of {ROTATIONS}, got {rotate!r}")
        for name, p in (("drop_slice_prob", drop_slice_prob), ("shift_slice_prob", shift_slice_prob)):
            if not 0.0 <= p <= 1.0:
                raise ValueError(f"{name} must be a probability in [0, 1], got {p}")
        if shift_magnitude < 0:
            raise ValueError(f"shift_magnitude must be >= 0 voxels, got {shift_magnitude}")
        if noise_scale < 0.0:
            raise ValueError(f"noise_scale must be >= 0, got {noise_scale}")
        if not image_keys:
            raise ValueError("image_keys is empty, so no augmentation could ever apply")
        geometric = rotate != "none" or (shift_slice_prob > 0 and shift_magnitude > 0)
        if geometric and sample_axes is None:
            raise ValueError(
                "rotation and section shifting need the dataset's axis order (sample_axes), but "
                "this dataset declares none; configure only intensity/noise, or declare a layout"
            )
        if rotate == "inplane" and sample_axes is not None and SECTION_AXIS not in sample_axes:
            raise ValueError(
                f"rotate='inplane' holds the sectioning axis {SECTION_AXIS!r} fixed, but the layout "
                f"{sample_axes!r} has none; use rotate='full'"
            )
        self.rotate = rotate
        self.drop_slice_prob = drop_slice_prob
        self.shift_slice_prob = shift_slice_prob
        self.shift_magnitude = shift_magnitude
        self.intensity = intensity
        self.mul_intensity = mul_intensity
        self.add_intensity = add_intensity
        self.noise_scale = noise_scale
        self.sample_axes = sample_axes
        self.image_keys = tuple(image_keys)
        self.label_keys = tuple(label_keys)

    def _dims_for(self, key: str) -> tuple[int, ...]:
        assert self.sample_axes is not None
        layout = self.sample_axes if key in self.image_keys else self.sample_axes.replace("c", "")
        return spatial_dims(layout)

    def _section_slot(self) -> int:
        assert self.sample_axes is not None
        return [a for a in self.sample_axes if a in SPATIAL_AXES].index(SECTION_AXIS)

    def _check_voxels(self, sample: dict[str, Any]) -> None:
        """Axes a rotation exchanges must share a voxel size (checked when `pixel_size` is known)."""
        pixel_size = sample.get("pixel_size")
        if pixel_size is None:
            return
        rank = len(self._dims_for(self.image_keys[0]))
        sizes = torch.as_tensor(pixel_size, dtype=torch.float64).reshape(-1, rank)
        slots = [s for s in range(rank) if self.rotate == "full" or s != self._section_slot()]
        held = sizes[:, slots]
        if not torch.allclose(held, held[:, :1], rtol=1e-6, atol=1e-9):
            raise ValueError(
                f"rotate={self.rotate!r} exchanges spatial slots {slots}, which need one voxel size, "
                f"but pixel_size={sizes.tolist()}; use rotate='inplane'"
            )

    @staticmethod
    def _coin(p: float = APPLY_PROB) -> bool:
        return bool(torch.rand(()).item() < p)

    @staticmethod
    def _present(sample: dict[str, Any], keys: tuple[str, ...]) -> list[str]:
        return [k for k in keys if k in sample and getattr(sample[k], "numel", lambda: 1)()]

    def __call__(self, sample: dict[str, Any]) -> dict[str, Any]:
        images = self._present(sample, self.image_keys)
        if not images:
            raise KeyError(
                f"no image key {self.image_keys} in the sample (keys {sorted(sample)}); "
                "augmentation would silently do nothing"
            )
        together = images + self._present(sample, self.label_keys)
        out = dict(sample)
        if self.rotate != "none":
            self._check_voxels(out)
            rotated = rot90(
                [out[k] for k in together],
                [self._dims_for(k) for k in together],
                fixed_slot=None if self.rotate == "full" else self._section_slot(),
            )
            out.update(zip(together, rotated, strict=True))
        if self.shift_slice_prob > 0 and self.shift_magnitude > 0 and self._coin():
            shifted = shift_sections(
                [out[k] for k in together],
                [self._dims_for(k) for k in together],
                self.shift_slice_prob,
                self.shift_magnitude,
            )
            out.update(zip(together, shifted, strict=True))
        if self.drop_slice_prob > 0 and self._coin():
            for k in images:
                out[k] = drop_sections(out[k], self._dims_for(k), self.drop_slice_prob)
        if self.intensity and self._coin():
            for k in images:
                out[k] = intensity_jitter(out[k], self.mul_intensity, self.add_intensity)
        if self.noise_scale > 0 and self._coin():
            for k in images:
                out[k] = additive_noise(out[k], self.noise_scale)
        return out
