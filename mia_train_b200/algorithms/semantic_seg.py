"""`semantic_seg`: per-voxel class prediction, 2-D or 3-D (reference `src/algorithms/semantic_seg.py:30-230`).

Encoder patch features -> 1x1 conv + GELU on the patch grid -> `VoxelHead` (separable upsampling,
3-wide conv, GELU, 1x1 conv to `num_classes`). Loss: cross-entropy with optional class weights and
`ignore_index`; metrics: pixel accuracy, mean IoU over the classes present in the batch, and their
count. On CUDA loss, argmax and the per-class histogram come from one fused kernel (no per-class
host loop). `checkpoint_decoder = True` recomputes `decoder_out` in backward (non-reentrant
checkpoint).
"""

from __future__ import annotations

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
            raise ValueError(f"num_classes must be at least 2, got {num_classes}")
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        self.input_key = input_key
        self.label_key = label_key
        self.num_classes = num_classes
        self.ignore_index = ignore_index
        self.checkpoint_decoder = checkpoint_decoder
        self.encoder = model
        self.spatial_rank = len([a for a in self.input_axes if a not in "lc"])
        if self.spatial_rank not in CONV:
            raise ValueError(
                f"axis order {self.input_axes!r} implies {self.spatial_rank} spatial axes; 2 or 3 are supported"
            )
        conv = CONV[self.spatial_rank]
        embed_dim = int(model.embed_dim)
        self.decoder = nn.Sequential(conv(embed_dim, decoder_hidden_dim, kernel_size=1), nn.GELU())
        self.decoder_out = VoxelHead(
            conv(decoder_hidden_dim, decoder_hidden_dim, kernel_size=3, padding=1),
            nn.GELU(),
            conv(decoder_hidden_dim, num_classes, kernel_size=1),
            mode=INTERPOLATION[self.spatial_rank],
        )
        weights = None if class_weights is None else torch.tensor(list(class_weights), dtype=torch.float32)
        if weights is not None and weights.numel() != num_classes:
            raise ValueError(f"class_weights has {weights.numel()} entries but num_classes={num_classes}")
        self.register_buffer("class_weights", weights, persistent=weights is not None)

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return (self.decoder_out,)

    def _prepare_labels(self, labels: torch.Tensor) -> torch.Tensor:
        label_axes = self.input_axes.replace("c", "")
        if labels.dim() != len(label_axes) + 1:
            raise ValueError(
                f"labels imply a {len(label_axes) + 1}-D batch from axis order {label_axes!r}, got {tuple(labels.shape)}"
            )
        level_dim = label_axes.index("l") + 1
        if labels.shape[level_dim] != 1:
            raise ValueError(
                f"semantic targets are single-scale, but this batch carries {labels.shape[level_dim]} levels "
                f"(shape {tuple(labels.shape)})"
            )
        return labels.squeeze(level_dim).long()

    def logits(self, volumes: torch.Tensor) -> torch.Tensor:
        """(B, C, *spatial) -> (B, num_classes, *spatial) class scores."""
        tokens, grid = self.encoder.patch_features(volumes)
        b, n, c = tokens.shape
        expected = 1
        for g in grid:
            expected *= g
        if n != expected:
            raise ValueError(f"encoder returned {n} tokens but its grid {grid} holds {expected}")
        x = self.decoder(tokens.transpose(1, 2).reshape(b, c, *grid))
        size = tuple(volumes.shape[2:])
        if self.checkpoint_decoder and torch.is_grad_enabled():
            return checkpoint(self.decoder_out, x, size, use_reentrant=False)
        return self.decoder_out(x, size)

    def _step(self, batch: Any) -> dict[str, torch.Tensor]:
        if self.label_key not in batch:
            raise KeyError(f"batch has no {self.label_key!r} key; got keys {sorted(batch)}")
        volumes = self.encoder.prepare_input(batch[self.input_key], self.input_axes)
        labels = self._prepare_labels(batch[self.label_key])
        if labels.shape[0] != volumes.shape[0] or labels.shape[1:] != volumes.shape[2:]:
            raise ValueError(f"label crop {tuple(labels.shape)} does not match the image crop {tuple(volumes.shape)}")
        scores = self.logits(volumes)
        return semantic_ce(scores, labels, self.class_weights, self.ignore_index)

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step(batch)
