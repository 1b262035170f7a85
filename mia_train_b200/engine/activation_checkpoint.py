"""Activation checkpointing of declared regions (reference `src/engine/activation_checkpoint.py:39-96`).

Models and algorithms declare their regions through `checkpointable_modules()`; the engine wraps
exactly those instances (identity match, so a block nested in one already wrapped is not paid for
twice) with non-reentrant `checkpoint_wrapper`, before sharding. Nothing declared is an error.
"""

from __future__ import annotations

import logging

import torch.nn as nn
from torch.distributed.algorithms._checkpoint.checkpoint_wrapper import CheckpointImpl, checkpoint_wrapper

from ..algorithms.base import BaseAlgorithm
from ..models.base import BaseModel

logger = logging.getLogger(__name__)


def checkpointable_targets(root: nn.Module) -> list[nn.Module]:
    targets: list[nn.Module] = []
    seen: set[int] = set()
    for module in root.modules():
        if not isinstance(module, (BaseModel, BaseAlgorithm)):
            continue
        for target in module.checkpointable_modules():
            if id(target) not in seen:
                seen.add(id(target))
                targets.append(target)
    return targets


def apply_activation_checkpointing(root: nn.Module) -> int:
    targets = checkpointable_targets(root)
    if not targets:
        raise ValueError(
            f"activation_checkpointing is on, but nothing under {type(root).__name__} declares "
            "checkpointable_modules(); implement it on the model or algorithm, or turn it off"
        )
    _wrap_children(root, {id(t) for t in targets})
    logger.info("activation checkpointing: recomputing %d module(s)", len(targets))
    return len(targets)


def _wrap_children(module: nn.Module, wanted: set[int]) -> None:
    for name, child in list(module.named_children()):
        if id(child) in wanted:
            setattr(module, name, checkpoint_wrapper(child, checkpoint_impl=CheckpointImpl.NO_REENTRANT))
        else:
            _wrap_children(child, wanted)
