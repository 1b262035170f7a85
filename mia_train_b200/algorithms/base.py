"""Training-strategy contract (reference `src/algorithms/base.py:13-73`).

An algorithm wraps a model with masking, heads and the loss. `forward` aliases `training_step`, so
DDP's forward hooks enclose the whole step even when the strategy drives the model through methods
other than its `forward`.

New here: `after_optimizer_step(step)` is called by the engine after every optimizer step. The
reference defines a DINOv3 teacher EMA but never calls it from the engine
(`src/algorithms/dinov3_ssl.py:223-230`); this hook is how `dinov3` updates its teacher.
"""

from __future__ import annotations

import abc
from typing import TYPE_CHECKING, Any

import torch
import torch.nn as nn

if TYPE_CHECKING:
    from ..data.base import BaseDataset


class BaseAlgorithm(nn.Module, abc.ABC):
    def __init__(self, model: nn.Module, dataset: BaseDataset | None = None) -> None:
        super().__init__()
        self.model = model
        self.dataset = dataset

    @abc.abstractmethod
    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        """One training iteration; the result must contain a "loss" key."""

    @abc.abstractmethod
    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        """One validation iteration; returns metrics for this batch."""

    def sample_transform(self) -> Any | None:
        """Per-sample preprocessing to run in the dataloader workers (train and validation)."""
        return None

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        """The strategy's own regions worth recomputing in backward (e.g. its decoder blocks)."""
        return ()

    def after_optimizer_step(self, step: int) -> None:
        """Engine hook after each optimizer step (1-based `step` just completed)."""

    def forward(self, batch: Any) -> dict[str, torch.Tensor]:
        return self.training_step(batch)

    @staticmethod
    def resolve_input_axes(input_axes: str | None, dataset: BaseDataset | None) -> str:
        """The dataset's declared layout wins; an explicit, contradicting `input_axes` is an error."""
        declared = dataset.sample_axes if dataset is not None else None
        if input_axes is not None and declared is not None and input_axes != declared:
            raise ValueError(
                f"input_axes={input_axes!r} contradicts the dataset's sample_axes={declared!r}; drop "
                "input_axes and let the dataset define the layout"
            )
        axes = input_axes or declared
        if axes is None:
            raise ValueError(
                "cannot determine the sample axis order: pass input_axes or use a dataset that "
                "exposes sample_axes"
            )
        return axes
