"""Architecture contract (reference `src/models/base.py:11-128`).

A model declares, besides `forward` and `flops`: how to turn a dataset batch into its input
(`prepare_input`), per-patch features for dense heads (`patch_features`), methods other than
`forward` through which its parameters are used (`extra_forward_methods`, for FSDP2), blocks worth
recomputing or sharding separately (`checkpointable_modules`), LoRA target groups and parameters
that must stay trainable under LoRA, and an optional tensor-parallel plan.
"""

from __future__ import annotations

import abc
from typing import Any

import torch
import torch.nn as nn


class BaseModel(nn.Module, abc.ABC):
    @abc.abstractmethod
    def forward(self, *args: Any, **kwargs: Any) -> Any: ...

    @abc.abstractmethod
    def flops(self, input_shape: tuple[int, ...]) -> int:
        """Forward FLOPs for one input of `input_shape` (no batch dim); raise for shapes it cannot run."""

    def prepare_input(self, batch: torch.Tensor, axes: str) -> torch.Tensor:
        raise NotImplementedError(
            f"{type(self).__name__} does not implement prepare_input, so it cannot be driven by an "
            "algorithm that passes dataset-shaped batches through the model"
        )

    def patch_features(self, x: torch.Tensor) -> tuple[torch.Tensor, tuple[int, ...]]:
        raise NotImplementedError(
            f"{type(self).__name__} does not implement patch_features, so it cannot drive a dense head"
        )

    def extra_forward_methods(self) -> tuple[str, ...]:
        return ()

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return ()

    def lora_target_groups(self) -> dict[str, tuple[nn.Linear, ...]]:
        return {}

    def lora_required_trainable(self) -> tuple[str, ...]:
        return ()

    def num_parameters(self, trainable_only: bool = False) -> int:
        return sum(p.numel() for p in self.parameters() if not trainable_only or p.requires_grad)

    def tensor_parallel_plan(self) -> dict[str, Any] | None:
        """Module-path -> ParallelStyle plan for tensor parallelism; None means unsupported."""
        return None
