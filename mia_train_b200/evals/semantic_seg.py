"""`semantic_seg` evaluation: whole-volume inference by overlapping tiles, a 2-D-on-3-D orthoplane
mode, and dataset-wide confusion metrics.

Role and config interface of reference `src/evals/semantic_seg.py:53-298` (task name, keys,
metric names); the implementation is this framework's own.

* `tile_starts(extent, tile, overlap)` spreads the fewest tiles that keep at least `overlap` voxels
  of overlap evenly over the axis: the first tile starts at 0, the last ends at the edge, so every
  voxel is predicted with real context on both sides wherever the volume allows.
* `blend_weight(shape)` is a separable tent, the product over axes of `min(i, n - 1 - i) + 1`:
  small at a tile's faces, large at its centre, so overlapping tiles blend without seams.
* `TileBlender` sums weighted tile scores and the weights themselves; `tiled_logits` drives it over
  a batch of same-sized images. The sums live on the compute device when they fit in
  `device_budget_bytes` (default: half the free device memory -- 64 classes over a 500^3 volume is
  32 GB, which fits in HBM3e) and on the host otherwise.
* `orthoplane_logits` applies a 2-D predictor to every plane normal to x, y and z and averages the
  three score volumes.
* `ConfusionMatrix` accumulates (target, prediction) counts on the device; `metrics()` reports pixel
  accuracy, mean IoU and mean Dice over the classes present in the ground truth, and per-class IoU.
"""

from __future__ import annotations

import itertools
import math
from collections.abc import Callable, Sequence
from functools import reduce

import torch
import torch.nn as nn
import torch.utils.data as data

from .base import BaseEvalTask
from .registry import EvalRegistry

AXES = ("x", "y", "z")


def tile_starts(extent: int, tile: int, overlap: int) -> list[int]:
    """Origins of the tiles along one axis (see the module docstring)."""
    span = extent - tile
    if span <= 0:
        return [0]
    stride = max(1, tile - overlap)
    count = math.ceil(span / stride) + 1
    return [round(i * span / (count - 1)) for i in range(count)]


def blend_weight(shape: Sequence[int], device: torch.device) -> torch.Tensor:
    """Separable tent weight over a tile of `shape`."""
    ramps = []
    for axis, n in enumerate(shape):
        pos = torch.arange(n, device=device, dtype=torch.float32)
        ramp = torch.minimum(pos, (n - 1) - pos) + 1.0
        view = [1] * len(shape)
        view[axis] = n
        ramps.append(ramp.view(view))
    return reduce(torch.mul, ramps, torch.ones((), device=device))


def _pick_device(nbytes: int, device: torch.device, budget: int | None) -> torch.device:
    if device.type != "cuda":
        return torch.device("cpu")
    room = torch.cuda.mem_get_info(device)[0] // 2 if budget is None else budget
    return device if nbytes <= room else torch.device("cpu")


class TileBlender:
    """Weighted sum of overlapping tile predictions over `count` images of shape `spatial`."""

    def __init__(self, count: int, channels: int, spatial: Sequence[int], tile: Sequence[int],
                 device: torch.device) -> None:
        self.tile = tuple(tile)
        self.device = device
        self.scores = torch.zeros((count, channels, *spatial), device=device)
        self.weights = torch.zeros(tuple(spatial), device=device)
        self.kernel = blend_weight(self.tile, device)

    def window(self, corner: Sequence[int]) -> tuple[slice, ...]:
        return tuple(slice(c, c + t) for c, t in zip(corner, self.tile, strict=True))

    def cover(self, corners: Sequence[Sequence[int]]) -> None:
        for corner in corners:
            self.weights[self.window(corner)] += self.kernel

    def add(self, image: int, corner: Sequence[int], scores: torch.Tensor) -> None:
        self.scores[image][(slice(None), *self.window(corner))] += scores.to(self.device) * self.kernel

    def result(self) -> torch.Tensor:
        return self.scores / self.weights.clamp_min(1e-8)


@torch.no_grad()
def tiled_logits(
    predict: Callable[[torch.Tensor], torch.Tensor],
    images: torch.Tensor,
    tile: Sequence[int],
    overlap: int,
    num_classes: int,
    device: torch.device,
    batch_size: int = 1,
    device_budget_bytes: int | None = None,
) -> torch.Tensor:
    """(N, *spatial) images -> (N, num_classes, *spatial) blended class scores."""
    count, spatial = images.shape[0], tuple(images.shape[1:])
    tile = tuple(min(t, s) for t, s in zip(tile, spatial, strict=True))
    nbytes = 4 * count * num_classes * math.prod(spatial)
    blender = TileBlender(count, num_classes, spatial, tile, _pick_device(nbytes, device, device_budget_bytes))
    corners = list(itertools.product(*(tile_starts(s, t, overlap) for s, t in zip(spatial, tile, strict=True))))
    blender.cover(corners)
    work = list(itertools.product(range(count), corners))
    for lo in range(0, len(work), batch_size):
        part = work[lo:lo + batch_size]
        windows = torch.stack([images[i][blender.window(c)] for i, c in part])[:, None]
        scores = predict(windows.to(device, non_blocking=True)).float()
        for (i, c), s in zip(part, scores, strict=True):
            blender.add(i, c, s)
    return blender.result()


@torch.no_grad()
def orthoplane_logits(
    predict: Callable[[torch.Tensor], torch.Tensor],
    volume: torch.Tensor,
    tile: Sequence[int],
    overlap: int,
    num_classes: int,
    device: torch.device,
    batch_size: int = 8,
    axes: Sequence[str] = AXES,
    device_budget_bytes: int | None = None,
) -> torch.Tensor:
    """(X, Y, Z) volume and a 2-D predictor -> (num_classes, X, Y, Z) scores averaged over plane axes."""
    total: torch.Tensor | None = None
    for name in axes:
        axis = AXES.index(name)
        stack = volume.movedim(axis, 0)  # planes normal to `axis`
        scores = tiled_logits(predict, stack, tile, overlap, num_classes, device, batch_size, device_budget_bytes)
        scores = scores.permute(1, 0, 2, 3).movedim(1, axis + 1)  # (C, X, Y, Z)
        total = scores if total is None else total + scores.to(total.device)
    if total is None:
        raise ValueError("orthoplane_logits needs at least one axis")
    return total / len(axes)


class ConfusionMatrix:
    """counts[t, p]: voxels of true class t predicted as p."""

    def __init__(self, num_classes: int, device: torch.device | str = "cpu") -> None:
        self.num_classes = num_classes
        self.counts = torch.zeros((num_classes, num_classes), dtype=torch.int64, device=device)

    def update(self, predicted: torch.Tensor, target: torch.Tensor, ignore_index: int) -> None:
        t = target.reshape(-1).to(self.counts.device)
        p = predicted.reshape(-1).to(self.counts.device)
        keep = t != ignore_index
        flat = t[keep].long() * self.num_classes + p[keep].long()
        self.counts.view(-1).index_add_(0, flat, torch.ones_like(flat))

    def metrics(self) -> dict[str, float]:
        c = self.counts.cpu().double()
        hits = torch.diagonal(c)
        truth, guess = c.sum(dim=1), c.sum(dim=0)
        present = truth > 0

        def ratio(num: torch.Tensor, den: torch.Tensor) -> torch.Tensor:
            return torch.where(den > 0, num / den.clamp_min(1.0), torch.zeros_like(den))

        iou = ratio(hits, truth + guess - hits)
        dice = ratio(2.0 * hits, truth + guess)
        report = {
            "pixel_accuracy": float(hits.sum() / c.sum().clamp_min(1.0)),
            "mean_iou": float(iou[present].mean()) if bool(present.any()) else 0.0,
            "mean_dice": float(dice[present].mean()) if bool(present.any()) else 0.0,
            "classes_present": float(present.sum()),
        }
        report.update({f"iou/class_{k}": float(iou[k]) for k in present.nonzero().flatten().tolist()})
        return report


@EvalRegistry.register("semantic_seg")
class SemanticSegmentationEval(BaseEvalTask):
    def __init__(
        self,
        num_classes: int = 64,
        tile: Sequence[int] = (256, 256, 256),
        overlap: int = 32,
        mode: str = "native",
        batch_size: int = 1,
        ignore_index: int = -1,
        axes: Sequence[str] = AXES,
        device: str | None = None,
        device_budget_bytes: int | None = None,
    ) -> None:
        super().__init__()
        if mode not in ("native", "orthoplane"):
            raise ValueError(f"semantic_seg eval: mode {mode!r} is neither 'native' nor 'orthoplane'")
        if overlap < 0:
            raise ValueError(f"semantic_seg eval: overlap {overlap} is negative")
        if not set(axes) <= set(AXES):
            raise ValueError(f"semantic_seg eval: axes {list(axes)} must be taken from x, y and z")
        self.num_classes = num_classes
        self.tile = tuple(int(t) for t in tile)
        self.overlap = overlap
        self.mode = mode
        self.batch_size = batch_size
        self.ignore_index = ignore_index
        self.axes = tuple(axes)
        self.device = device
        self.device_budget_bytes = device_budget_bytes

    def _scores(self, predict: Callable[[torch.Tensor], torch.Tensor], image: torch.Tensor,
                device: torch.device) -> torch.Tensor:
        if self.mode == "orthoplane":
            return orthoplane_logits(predict, image, self.tile, self.overlap, self.num_classes, device,
                                     self.batch_size, self.axes, self.device_budget_bytes)
        return tiled_logits(predict, image[None], self.tile, self.overlap, self.num_classes, device,
                            self.batch_size, self.device_budget_bytes)[0]

    def evaluate(self, model: nn.Module, dataloader: data.DataLoader) -> dict[str, float]:
        if not callable(getattr(model, "logits", None)):
            raise TypeError(f"semantic_seg eval needs a model with a `logits` method; {type(model).__name__} has none")
        rank = int(model.spatial_rank)
        if self.mode == "orthoplane" and rank != 2:
            raise ValueError(f"orthoplane mode slices volumes into 2-D planes; the model is {rank}-D")
        if len(self.tile) != rank:
            raise ValueError(f"tile {self.tile} has {len(self.tile)} sizes for a {rank}-D model")
        device = torch.device(self.device or ("cuda" if torch.cuda.is_available() else "cpu"))
        model.eval().to(device)
        confusion = ConfusionMatrix(self.num_classes, device)
        for batch in dataloader:
            for image, label in zip(batch["img"][:, 0, 0], batch["label"][:, 0].long(), strict=True):
                confusion.update(self._scores(model.logits, image, device).argmax(0), label, self.ignore_index)
        return confusion.metrics()
