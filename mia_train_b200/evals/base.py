"""Evaluation-task contract (reference `src/evals/base.py`): `evaluate(model, dataloader) -> metrics`."""

from __future__ import annotations

import abc

import torch.nn as nn
import torch.utils.data as data


class BaseEvalTask(nn.Module, abc.ABC):
    @abc.abstractmethod
    def evaluate(self, model: nn.Module, dataloader: data.DataLoader) -> dict[str, float]:
        """Run the evaluation loop against `model`; returns metric name -> value."""
