"""`semantic_seg`: a class score for every voxel (2-D or 3-D inputs).

Interface of reference `src/algorithms/semantic_seg.py:30-230` (registry name, constructor keys and
the parameter names `decoder.0` / `decoder_out.*`, which checkpoints depend on); the code is this
framework's own.

Encoder patch features (B, N, C) are laid back onto the patch grid, mixed by a 1x1 convolution +
GELU (`decoder`), then `VoxelHead` (`decoder_out`) upsamples them separably to voxel resolution
and applies a 3-wide convolution, GELU and a 1x1 convolution to `num_classes` scores. The loss is
cross-entropy with optional class weights and an `ignore_index`; metrics are pixel accuracy, mean
IoU over the classes present in the batch, and that count. On CUDA one fused kernel produces the
loss, the argmax and the per-class histogram (`ops.dense_loss.semantic_ce`). With
`checkpoint_decoder = True` the voxel-resolution head is recomputed in backward instead of kept.
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn as nn
from torch.utils.checkpoint import checkpoint

from ..data.base import BaseDataset
from ..layers.common.dense_heads import CONV, INTERPOLATION, VoxelHead
from ..ops.dense_loss import semantic_ce
from .base import BaseAlgorithm
from .registry import AlgorithmRegistry


@AlgorithmRegistry.register("semantic_seg")
class SemanticSegmentation(BaseAlgorithm):
    class_weights: torch.Tensor | None

    def __init__(
        self,
        model: nn.Module,
        dataset: BaseDataset | None = None,
        input_axes: str | None = None,
        input_key: str = "img",
        label_key: str = "label",
        num_classes: int = 64,
        decoder_hidden_dim: int = 128,
        ignore_index: int = -1,
        class_weights: tuple[float, ...] | list[float] | None = None,
        checkpoint_decoder: bool = False,
    ) -> None:
        super().__init__(model, dataset)
        if num_classes < 2:
            raise ValueError(f"semantic_seg: num_classes = {num_classes}; at least two classes are needed")
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        spatial = [a for a in self.input_axes if a not in "lc"]
        if len(spatial) not in CONV:
            raise ValueError(f"semantic_seg: axes {self.input_axes!r} have {len(spatial)} spatial axes; "
                             "only 2-D and 3-D inputs are supported")
        self.spatial_rank = len(spatial)
        self.input_key, self.label_key = input_key, label_key
        self.num_classes, self.ignore_index = num_classes, ignore_index
        self.checkpoint_decoder = checkpoint_decoder
        self.encoder = model
        # labels carry the image axes minus the channel axis; the level axis must have length 1
        self._label_axes = self.input_axes.replace("c", "")
        conv = CONV[self.spatial_rank]
        width = int(model.embed_dim)
        self.decoder = nn.Sequential(conv(width, decoder_hidden_dim, kernel_size=1), nn.GELU())
        self.decoder_out = VoxelHead(
            conv(decoder_hidden_dim, decoder_hidden_dim, kernel_size=3, padding=1),
            nn.GELU(),
            conv(decoder_hidden_dim, num_classes, kernel_size=1),
            mode=INTERPOLATION[self.spatial_rank],
        )
        weights = None
        if class_weights is not None:
            weights = torch.as_tensor(list(class_weights), dtype=torch.float32)
            if weights.numel() != num_classes:
                raise ValueError(f"semantic_seg: {weights.numel()} class_weights for {num_classes} classes")
        self.register_buffer("class_weights", weights, persistent=weights is not None)

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return (self.decoder_out,)

    def _prepare_labels(self, labels: torch.Tensor) -> torch.Tensor:
        """(B, [L=1,] *spatial) in the configured axis order -> (B, *spatial) int64."""
        want = len(self._label_axes) + 1
        if labels.dim() != want:
            raise ValueError(f"semantic_seg: labels of shape {tuple(labels.shape)} do not have the {want} dims of "
                             f"a batch in axis order {self._label_axes!r}")
        level = 1 + self._label_axes.index("l")
        if labels.size(level) != 1:
            raise ValueError(f"semantic_seg: labels have {labels.size(level)} levels; targets are single-scale")
        return labels.squeeze(level).long()

    def logits(self, volumes: torch.Tensor) -> torch.Tensor:
        """(B, C, *spatial) -> (B, num_classes, *spatial) class scores."""
        tokens, grid = self.encoder.patch_features(volumes)
        batch, count, width = tokens.shape
        if count != math.prod(grid):
            raise ValueError(f"semantic_seg: the encoder gave {count} tokens for a patch grid {tuple(grid)}")
        features = self.decoder(tokens.transpose(1, 2).reshape(batch, width, *grid))
        size = tuple(volumes.shape[2:])
        if self.checkpoint_decoder and torch.is_grad_enabled():
            return checkpoint(self.decoder_out, features, size, use_reentrant=False)
        return self.decoder_out(features, size)

    def _step(self, batch: Any) -> dict[str, torch.Tensor]:
        if self.label_key not in batch:
            raise KeyError(f"semantic_seg: the batch has no {self.label_key!r} entry (keys: {sorted(batch)})")
        volumes = self.encoder.prepare_input(batch[self.input_key], self.input_axes)
        labels = self._prepare_labels(batch[self.label_key])
        if labels.shape != (volumes.shape[0], *volumes.shape[2:]):
            raise ValueError(f"semantic_seg: label crop {tuple(labels.shape)} and image crop "
                             f"{tuple(volumes.shape)} disagree")
        return semantic_ce(self.logits(volumes), labels, self.class_weights, self.ignore_index)

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)
