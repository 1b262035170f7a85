"""Affinity targets from instance labels (reference `src/algorithms/affinity/targets.py:27-281`).

* `affinity_offsets(rank, long_range)` -- the default 2*rank channels: +1 along each axis, then
  +long_range along each axis, in the batch's spatial axis order.
* `offset_preset(name)` -- named offset lists; `"nisb12"` is 3 nearest-neighbour offsets plus long
  range offsets 3, 6 and 9 along each axis (12 channels, offsets up to 9 voxels).
* `affinities_from_labels` -- bool (target, mask): a pair is affine when both voxels carry the
  same positive id; the mask drops pairs touching `ignore_index` and the border slab each offset
  shifts in from.
* `relabel_connected` -- splits every id into its 6-connected pieces on the tensor's device by
  root hooking plus pointer jumping (data-dependent rounds, each ending in a host check).
* `relabel_connected_host` -- the same partition from the native host union-find (two-pass
  raster labelling in C++); `SplitDisconnectedLabels` runs it per sample in dataloader workers,
  which is where the engine puts it. `cc3d` is not needed.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch

from ...ops.dense_loss import affinity_targets_reference, offset_slices

SHORT_RANGE = 1
LONG_RANGE = 10

_PRESETS: dict[str, tuple[tuple[int, int, int], ...]] = {
    "nisb12": tuple(
        tuple(d if i == axis else 0 for i in range(3))  # type: ignore[misc]
        for d in (1, 3, 6, 9)
        for axis in range(3)
    ),
}


def affinity_offsets(spatial_rank: int, long_range: int = LONG_RANGE) -> tuple[tuple[int, ...], ...]:
    offsets = []
    for distance in (SHORT_RANGE, long_range):
        for axis in range(spatial_rank):
            o = [0] * spatial_rank
            o[axis] = distance
            offsets.append(tuple(o))
    return tuple(offsets)


def offset_preset(name: str) -> tuple[tuple[int, ...], ...]:
    if name not in _PRESETS:
        raise KeyError(f"unknown affinity offset preset {name!r}; available: {sorted(_PRESETS)}")
    return _PRESETS[name]


def affinities_from_labels(
    labels: torch.Tensor, offsets: Sequence[Sequence[int]], ignore_index: int = -1
) -> tuple[torch.Tensor, torch.Tensor]:
    return affinity_targets_reference(labels, offsets, ignore_index)


def _adjacency(labels: torch.Tensor, foreground: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Flat index pairs of face-adjacent voxels sharing a positive id (no wrap-around)."""
    index = torch.arange(labels.numel(), device=labels.device).view(labels.shape)
    src, dst = [], []
    for axis in range(labels.ndim):
        if labels.shape[axis] < 2:
            continue
        lo = tuple(slice(0, -1) if i == axis else slice(None) for i in range(labels.ndim))
        hi = tuple(slice(1, None) if i == axis else slice(None) for i in range(labels.ndim))
        same = (labels[lo] == labels[hi]) & foreground[lo]
        src.append(index[lo][same])
        dst.append(index[hi][same])
    if not src:
        e = torch.empty(0, dtype=torch.int64, device=labels.device)
        return e, e
    return torch.cat(src), torch.cat(dst)


def relabel_connected(labels: torch.Tensor) -> torch.Tensor:
    """Each spatially connected run of an id gets its own id 1..K; background / negatives kept."""
    if labels.ndim < 1:
        raise ValueError(f"labels need at least one spatial axis, got shape {tuple(labels.shape)}")
    shape = labels.shape
    fg = labels > 0
    parent = torch.arange(labels.numel(), device=labels.device)
    src, dst = _adjacency(labels, fg)
    while src.numel() > 0:
        prev = parent.clone()
        rs, rd = parent[src], parent[dst]
        low = torch.minimum(rs, rd)
        parent.scatter_reduce_(0, rs, low, reduce="amin")
        parent.scatter_reduce_(0, rd, low, reduce="amin")
        while True:
            jumped = parent[parent]
            if torch.equal(jumped, parent):
                break
            parent = jumped
        if torch.equal(parent, prev):
            break
    _, dense = torch.unique(parent.view(shape), return_inverse=True)
    return torch.where(fg, dense.reshape(shape) + 1, labels.long())


def relabel_connected_host(labels: torch.Tensor) -> torch.Tensor:
    """`relabel_connected` on the host with the native union-find; returns int64 on `labels.device`."""
    from ...ops.dense_loss import connected_components

    return connected_components(labels).to(labels.device)


def cc3d_available() -> bool:
    """The host labeller is part of the native extension; kept for the reference's name."""
    try:
        from ...ops._native import native

        native()
        return True
    except Exception:  # noqa: BLE001
        return False


class SplitDisconnectedLabels:
    """Worker-side transform: split one sample's `(L, *spatial)` labels into connected pieces per level."""

    def __init__(self, label_key: str = "label") -> None:
        self.label_key = label_key

    def __call__(self, sample: dict[str, Any]) -> dict[str, Any]:
        if self.label_key not in sample:
            raise KeyError(
                f"no {self.label_key!r} in the sample (keys {sorted(sample)}); the affinity objective asked "
                "for its labels to be split into connected components in the dataloader"
            )
        labels = sample[self.label_key]
        out = dict(sample)
        out[self.label_key] = torch.stack([relabel_connected_host(level) for level in labels]).to(labels.dtype)
        return out


__all__ = [
    "LONG_RANGE",
    "SHORT_RANGE",
    "SplitDisconnectedLabels",
    "affinities_from_labels",
    "affinity_offsets",
    "cc3d_available",
    "offset_preset",
    "offset_slices",
    "relabel_connected",
    "relabel_connected_host",
]
