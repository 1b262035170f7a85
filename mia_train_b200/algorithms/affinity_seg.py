"""`affinity_seg`: supervised instance segmentation by affinity prediction
(reference `src/algorithms/affinity_seg.py:43-329`).

Encoder patch features -> a dense head -> one logit per voxel and offset, trained with masked
BCE-with-logits against affinities derived from instance labels. Decoders: `"interpolate"`
(1x1 conv + GELU on the patch grid, then `VoxelHead`: separable upsampling, 3x3x3 conv, GELU,
1x1 conv) or `"subpixel"` (`SubPixelHead`). Offsets: the reference's 6 (`long_range`) by default,
a named preset (`offsets = "nisb12"`), or an explicit list of (dx, dy, dz) triples.

On CUDA the loss is the fused affinity kernel: targets and masks are recomputed from the labels
inside the loss and its gradient, never stored. Connected-component splitting goes to the
dataloader workers (native host union-find) when the engine asks for `sample_transform()`;
otherwise it runs on the device.

Under sequence-parallel tensor parallelism (`split_decoder_over_tp`, default on) each TP rank
decodes its own share of the batch's samples after the encoder, and the loss is weighted by each
rank's share of the voxels; a per-replica batch smaller than the TP group decodes replicated.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch
import torch.nn as nn

from ..data.base import BaseDataset
from ..layers.common.dense_heads import SubPixelHead, VoxelHead
from ..ops.dense_loss import affinity_bce
from .affinity.targets import (
    LONG_RANGE,
    SplitDisconnectedLabels,
    affinity_offsets,
    offset_preset,
    relabel_connected,
)
from .base import BaseAlgorithm
from .registry import AlgorithmRegistry

SPATIAL_RANK = 3
DECODERS = ("interpolate", "subpixel")


def _resolve_offsets(offsets: str | Sequence[Sequence[int]] | None, long_range: int) -> tuple[tuple[int, ...], ...]:
    if offsets is None:
        return affinity_offsets(SPATIAL_RANK, long_range)
    if isinstance(offsets, str):
        return offset_preset(offsets)
    out = tuple(tuple(int(v) for v in o) for o in offsets)
    if not out or any(len(o) != SPATIAL_RANK for o in out):
        raise ValueError(f"offsets must be a non-empty list of {SPATIAL_RANK}-component offsets, got {offsets!r}")
    if any(all(v == 0 for v in o) for o in out):
        raise ValueError("a zero offset relates every voxel to itself and carries no information")
    return out


@AlgorithmRegistry.register("affinity_seg")
class AffinitySegmentation(BaseAlgorithm):
    def __init__(
        self,
        model: nn.Module,
        dataset: BaseDataset | None = None,
        input_axes: str | None = None,
        input_key: str = "img",
        label_key: str = "label",
        long_range: int = LONG_RANGE,
        offsets: str | Sequence[Sequence[int]] | None = None,
        decoder: str = "interpolate",
        decoder_hidden_dim: int = 64,
        decoder_readout_dim: int = 16,
        decoder_refine_depth: int = 2,
        decoder_zero_init_output: bool = True,
        ignore_index: int = -1,
        split_disconnected: bool = True,
        split_decoder_over_tp: bool = True,
    ) -> None:
        super().__init__(model, dataset)
        if long_range < 1:
            raise ValueError(f"long_range must be at least 1 voxel, got {long_range}")
        if decoder not in DECODERS:
            raise ValueError(f"decoder must be one of {DECODERS}, got {decoder!r}")
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        spatial = [a for a in self.input_axes if a not in "lc"]
        if spatial != ["x", "y", "z"]:
            raise ValueError(
                f"axis order {self.input_axes!r} gives spatial order {''.join(spatial)!r}; affinity channels are "
                'defined in x,y,z order, so the dataset must deliver x,y,z (e.g. output_axes "lcxyz")'
            )
        self.input_key = input_key
        self.label_key = label_key
        self.ignore_index = ignore_index
        self.split_disconnected = split_disconnected
        self.offsets = _resolve_offsets(offsets, long_range)
        self.decoder_kind = decoder
        self.encoder = model
        self._split_delegated = False
        # Under sequence-parallel TP the encoder's tokens are gathered on every TP rank; the voxel
        # decoder and the loss then run on this rank's share of the samples only (the encoder's
        # final norm and the decoder become partial-gradient parameters summed over the group).
        self.split_decoder_over_tp = split_decoder_over_tp
        self._post_gather_marked = False
        embed_dim = int(model.embed_dim)
        n_out = len(self.offsets)
        if decoder == "subpixel":
            patch = model.patch_size
            patch_size = (patch,) * SPATIAL_RANK if isinstance(patch, int) else tuple(patch)
            self.decoder: nn.Module = nn.Identity()
            self.decoder_out: nn.Module = SubPixelHead(
                embed_dim, patch_size, n_out, hidden=decoder_hidden_dim, readout=decoder_readout_dim,
                refine_depth=decoder_refine_depth, zero_init_output=decoder_zero_init_output,
            )
        else:
            self.decoder = nn.Sequential(nn.Conv3d(embed_dim, decoder_hidden_dim, kernel_size=1), nn.GELU())
            self.decoder_out = VoxelHead(
                nn.Conv3d(decoder_hidden_dim, decoder_hidden_dim, kernel_size=3, padding=1),
                nn.GELU(),
                nn.Conv3d(decoder_hidden_dim, n_out, kernel_size=1),
                mode="trilinear",
            )

    def sample_transform(self) -> SplitDisconnectedLabels | None:
        if not self.split_disconnected:
            return None
        self._split_delegated = True
        return SplitDisconnectedLabels(self.label_key)

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return (self.decoder_out,)

    def _prepare_labels(self, labels: torch.Tensor) -> torch.Tensor:
        label_axes = self.input_axes.replace("c", "")
        if labels.dim() != len(label_axes) + 1:
            raise ValueError(
                f"labels imply a {len(label_axes) + 1}-D batch from axis order {label_axes!r}, got "
                f"{tuple(labels.shape)}"
            )
        level_dim = label_axes.index("l") + 1
        if labels.shape[level_dim] != 1:
            raise ValueError(
                f"affinity targets are single-scale, but this batch carries {labels.shape[level_dim]} levels on "
                f"axis 'l' (shape {tuple(labels.shape)})"
            )
        return labels.squeeze(level_dim).long()

    def _decode(self, tokens: torch.Tensor, grid: tuple[int, ...], size: Sequence[int]) -> torch.Tensor:
        b, n, c = tokens.shape
        expected = 1
        for g in grid:
            expected *= g
        if n != expected:
            raise ValueError(f"encoder returned {n} tokens but its grid {grid} holds {expected}")
        x = tokens.transpose(1, 2).reshape(b, c, *grid)
        x = self.decoder(x)
        return self.decoder_out(x, tuple(size))

    def _step(self, batch: Any) -> dict[str, torch.Tensor]:
        if self.label_key not in batch:
            raise KeyError(f"batch has no {self.label_key!r} key; got keys {sorted(batch)}")
        volumes = self.encoder.prepare_input(batch[self.input_key], self.input_axes)
        labels = self._prepare_labels(batch[self.label_key])
        if labels.shape[0] != volumes.shape[0] or labels.shape[1:] != volumes.shape[2:]:
            raise ValueError(
                f"label crop {tuple(labels.shape)} does not match the image crop {tuple(volumes.shape)}"
            )
        sp = getattr(self.encoder, "_sequence_parallel", None)
        split = sp is not None and self.split_decoder_over_tp and volumes.shape[0] >= sp.world
        if sp is not None and self.split_decoder_over_tp and not split and self._post_gather_marked:
            # the decoder's gradients are summed over the group once it has been split: a replicated
            # decode now would count them once per rank
            raise ValueError(
                f"a batch of {volumes.shape[0]} is smaller than the tensor-parallel group ({sp.world}) after "
                "earlier batches split the decoder over it; keep the per-replica batch at least the TP size"
            )
        # a per-replica batch smaller than the TP group decodes replicated on every TP rank
        part = sp.sample_slice(volumes.shape[0]) if split else None
        if part is not None:
            self._mark_post_gather(sp)
            sp.split_samples = True
        try:
            with torch.profiler.record_function("encoder"):
                tokens, grid = self.encoder.patch_features(volumes)
        finally:
            if part is not None:
                sp.split_samples = False
        if part is not None:
            tokens, labels = tokens[part], labels[part]
        with torch.profiler.record_function("decoder"):
            logits = self._decode(tokens, grid, volumes.shape[2:])
        if self.split_disconnected and not self._split_delegated:
            with torch.profiler.record_function("relabel_connected"):
                labels = torch.stack([relabel_connected(s) for s in labels])
        with torch.profiler.record_function("affinity_loss"):
            out = affinity_bce(logits, labels, self.offsets, self.ignore_index)
        return self._combine_over_tp(out, logits.numel(), sp) if part is not None else out

    def _mark_post_gather(self, sp: Any) -> None:
        if self._post_gather_marked:
            return
        from ..parallel.sequence_parallel import mark_post_gather_params

        mods = [self.decoder, self.decoder_out]
        for name in ("norm", "cls_norm", "local_cls_norm"):
            mod = getattr(self.encoder, name, None)
            if isinstance(mod, nn.Module):
                mods.append(mod)
        mark_post_gather_params(mods, sp.group)
        self._post_gather_marked = True

    @staticmethod
    def _combine_over_tp(out: dict[str, torch.Tensor], numel: int, sp: Any) -> dict[str, torch.Tensor]:
        """Every TP rank scored its own samples: weight each rank's masked-mean loss by its share of
        the group's unmasked voxels (so the ranks' gradients sum to the whole batch's), and report
        the whole batch's loss and metrics on every rank."""
        import torch.distributed as dist

        count = out["masked_fraction"].detach().float() * numel
        stats = torch.stack([count, out["loss"].detach().float() * count, out["affinity_accuracy"].float() * count,
                             out["target_positive_rate"].float() * count, out["boundary_accuracy"].float() * count,
                             torch.full_like(count, float(numel))])
        dist.all_reduce(stats, group=sp.group)
        total = stats[0].clamp_min(1.0)
        weighted = out["loss"] * (count / total)
        whole = stats[1] / total
        return {
            "loss": weighted + (whole - weighted).detach(),  # the batch's value, this rank's gradient
            "affinity_accuracy": stats[2] / total,
            "target_positive_rate": stats[3] / total,
            "boundary_accuracy": stats[4] / total,  # voxel-weighted across ranks
            "masked_fraction": stats[0] / stats[5],
        }

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)
