"""Moving collated batches onto the training device (reference `src/utils/device.py:9-22`)."""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

import torch


def move_to_device(batch: Any, device: torch.device) -> Any:
    """Recursively copy every tensor in `batch` to `device` without blocking the host.

    Dicts, lists and tuples are walked; anything else (strings, ints, metadata) passes through.
    """
    if isinstance(batch, torch.Tensor):
        return batch.to(device, non_blocking=True)
    if isinstance(batch, Mapping):
        return {key: move_to_device(value, device) for key, value in batch.items()}
    if isinstance(batch, (list, tuple)):
        return type(batch)(move_to_device(value, device) for value in batch)
    return batch


def pin_batch(batch: Any) -> Any:
    """Page-lock every CPU tensor of `batch` so its host->device copy can run asynchronously."""
    if isinstance(batch, torch.Tensor):
        return batch.pin_memory() if batch.device.type == "cpu" and not batch.is_pinned() else batch
    if isinstance(batch, Mapping):
        return {key: pin_batch(value) for key, value in batch.items()}
    if isinstance(batch, (list, tuple)):
        return type(batch)(pin_batch(value) for value in batch)
    return batch


def tensor_bytes(batch: Any) -> int:
    """Total bytes held by the tensors of a (nested) batch."""
    if isinstance(batch, torch.Tensor):
        return batch.numel() * batch.element_size()
    if isinstance(batch, Mapping):
        return sum(tensor_bytes(value) for value in batch.values())
    if isinstance(batch, (list, tuple)):
        return sum(tensor_bytes(value) for value in batch)
    return 0
