"""`semantic_seg` evaluation: tiled whole-volume inference, orthoplane 2-D-on-3-D, confusion metrics
(reference `src/evals/semantic_seg.py:53-298`).

* `tile_starts` -- window origins with the requested overlap; the last window is pulled back to
  end at the volume's edge, so every voxel is predicted from real context.
* `blend_weight` -- per-tile weight, the product over axes of `min(i, n - 1 - i) + 1` (low at the
  faces, high at the centre), so overlapping tiles blend without seams.
* `tiled_logits` -- blended class scores for a batch of same-shaped images. The accumulator lives
  on the compute device when it fits in `device_budget_bytes` (default: half of the free device
  memory; 64 classes over a 500^3 volume is 32 GB, which an HBM3e part holds) and on the host
  otherwise; the blend-weight sum is accumulated once per tiling, not per image.
* `orthoplane_logits` -- a 2-D predictor over every plane normal to x, y and z, averaged in score
  space.
* `ConfusionMatrix` -- dataset-wide counts (`bincount` on the device); pixel accuracy, mean IoU
  and mean Dice over the classes present in the ground truth, and per-class IoU.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
import torch.nn as nn
import torch.utils.data as data

from .base import BaseEvalTask
from .registry import EvalRegistry

AXES = ("x", "y", "z")


def tile_starts(extent: int, tile: int, overlap: int) -> list[int]:
    if tile >= extent:
        return [0]
    stride = max(tile - overlap, 1)
    starts = list(range(0, extent - tile + 1, stride))
    if starts[-1] != extent - tile:
        starts.append(extent - tile)
    return starts


def blend_weight(shape: Sequence[int], device: torch.device) -> torch.Tensor:
    w = torch.ones(tuple(shape), device=device)
    for axis, n in enumerate(shape):
        i = torch.arange(n, device=device)
        ramp = (torch.minimum(i, n - 1 - i) + 1).float()
        w = w * ramp.reshape([-1 if k == axis else 1 for k in range(len(shape))])
    return w


def _accumulator_device(nbytes: int, device: torch.device, budget: int | None) -> torch.device:
    if device.type != "cuda":
        return torch.device("cpu")
    if budget is None:
        free, _ = torch.cuda.mem_get_info(device)
        budget = free // 2
    return device if nbytes <= budget else torch.device("cpu")


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
    """(N, *spatial) -> (N, num_classes, *spatial) blended scores (on the accumulator's device)."""
    spatial = tuple(images.shape[1:])
    tile = tuple(min(t, s) for t, s in zip(tile, spatial, strict=True))
    nbytes = 4 * images.shape[0] * num_classes * int(torch.tensor(spatial).prod())
    acc_dev = _accumulator_device(nbytes, device, device_budget_bytes)
    total = torch.zeros((images.shape[0], num_classes, *spatial), dtype=torch.float32, device=acc_dev)
    weight = torch.zeros(spatial, dtype=torch.float32, device=acc_dev)
    single = blend_weight(tile, acc_dev)
    corners: list[tuple[int, ...]] = [()]
    for s, t in zip(spatial, tile, strict=True):
        corners = [c + (o,) for c in corners for o in tile_starts(s, t, overlap)]

    def window(c: tuple[int, ...]) -> tuple[slice, ...]:
        return tuple(slice(o, o + t) for o, t in zip(c, tile, strict=True))

    for c in corners:
        weight[window(c)] += single
    jobs = [(n, c) for n in range(images.shape[0]) for c in corners]
    for begin in range(0, len(jobs), batch_size):
        chunk = jobs[begin : begin + batch_size]
        batch = torch.stack([images[n][window(c)] for n, c in chunk])
        scores = predict(batch[:, None].to(device, non_blocking=True)).float().to(acc_dev)
        for (n, c), s in zip(chunk, scores, strict=True):
            total[n][(slice(None), *window(c))] += s * single
    return total / weight.clamp_min(1e-8)


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
    """(X, Y, Z) volume + 2-D predictor -> (num_classes, X, Y, Z) scores averaged over the plane axes."""
    acc = None
    for axis in axes:
        k = AXES.index(axis)
        planes = volume.movedim(k, 0)
        s = tiled_logits(predict, planes, tile, overlap, num_classes, device, batch_size, device_budget_bytes)
        s = s.movedim(1, 0).movedim(1, k + 1)
        acc = s if acc is None else acc + s.to(acc.device)
    assert acc is not None
    return acc / len(axes)


class ConfusionMatrix:
    def __init__(self, num_classes: int, device: torch.device | str = "cpu") -> None:
        self.num_classes = num_classes
        self.counts = torch.zeros((num_classes, num_classes), dtype=torch.int64, device=device)

    def update(self, predicted: torch.Tensor, target: torch.Tensor, ignore_index: int) -> None:
        predicted = predicted.to(self.counts.device)
        target = target.to(self.counts.device)
        valid = target != ignore_index
        idx = target[valid].flatten().long() * self.num_classes + predicted[valid].flatten().long()
        self.counts += torch.bincount(idx, minlength=self.num_classes**2).reshape(self.num_classes, self.num_classes)

    def metrics(self) -> dict[str, float]:
        c = self.counts.double().cpu()
        tp = c.diag()
        actual, pred = c.sum(1), c.sum(0)
        union = actual + pred - tp
        present = actual > 0
        iou = torch.where(union > 0, tp / union.clamp_min(1), torch.zeros_like(union))
        dice = torch.where(actual + pred > 0, 2 * tp / (actual + pred).clamp_min(1), torch.zeros_like(union))
        out = {
            "pixel_accuracy": float(tp.sum() / c.sum().clamp_min(1)),
            "mean_iou": float(iou[present].mean()) if present.any() else 0.0,
            "mean_dice": float(dice[present].mean()) if present.any() else 0.0,
            "classes_present": float(present.sum()),
        }
        for k in torch.nonzero(present).flatten().tolist():
            out[f"iou/class_{k}"] = float(iou[k])
        return out


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
            raise ValueError(f"mode must be 'native' or 'orthoplane', got {mode!r}")
        if overlap < 0:
            raise ValueError(f"overlap must be >= 0, got {overlap}")
        unknown = sorted(set(axes) - set(AXES))
        if unknown:
            raise ValueError(f"axes must be drawn from x, y, z; got {unknown}")
        self.num_classes = num_classes
        self.tile = tuple(int(t) for t in tile)
        self.overlap = overlap
        self.mode = mode
        self.batch_size = batch_size
        self.ignore_index = ignore_index
        self.axes = tuple(axes)
        self.device = device
        self.device_budget_bytes = device_budget_bytes

    def evaluate(self, model: nn.Module, dataloader: data.DataLoader) -> dict[str, float]:
        if not hasattr(model, "logits"):
            raise TypeError(f"{type(model).__name__} has no `logits` method; evaluate a semantic_seg algorithm")
        rank = int(model.spatial_rank)
        if self.mode == "orthoplane" and rank != 2:
            raise ValueError(f"mode='orthoplane' feeds 2-D planes, but this algorithm is {rank}-D")
        if len(self.tile) != rank:
            raise ValueError(f"tile {self.tile} has {len(self.tile)} entries but the model is {rank}-D")
        device = torch.device(self.device or ("cuda" if torch.cuda.is_available() else "cpu"))
        model.eval().to(device)
        confusion = ConfusionMatrix(self.num_classes, device)

        def predict(windows: torch.Tensor) -> torch.Tensor:
            return model.logits(windows)

        for batch in dataloader:
            images = batch["img"][:, 0, 0]
            labels = batch["label"][:, 0].long()
            for image, label in zip(images, labels, strict=True):
                if self.mode == "orthoplane":
                    scores = orthoplane_logits(predict, image, self.tile, self.overlap, self.num_classes, device,
                                               self.batch_size, self.axes, self.device_budget_bytes)
                else:
                    scores = tiled_logits(predict, image[None], self.tile, self.overlap, self.num_classes, device,
                                          self.batch_size, self.device_budget_bytes)[0]
                confusion.update(scores.argmax(0), label, self.ignore_index)
        return confusion.metrics()
