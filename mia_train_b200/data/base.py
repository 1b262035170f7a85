"""The dataset contract every `[data]` implementation fulfils, and its dataloader.

Interface of reference `src/data/base.py:11-181` (the methods the engine calls); the code is this
framework's own.

* A dataset is built lazily on first use of `.dataset`, so per-sample transforms (augmentation,
  the algorithm's own `sample_transform`) can be attached first; once built, attaching is refused
  because samples already handed out would have skipped the transform. Transforms run in the order
  they were attached, inside the worker processes.
* The loader shards indices over the data-parallel ranks only (tensor-parallel peers read the same
  samples), drops the last partial batch (a short batch would change the step's shapes and, in
  graph mode, force a re-capture), pins host memory when worker processes produce the batches, and
  limits each worker to one intra-op thread so they do not compete with the host thread that
  launches kernels.
"""

from __future__ import annotations

import abc
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from torch.utils.data import DataLoader, Dataset, DistributedSampler

Transform = Callable[[dict[str, Any]], dict[str, Any]]


class _Chain:
    """Picklable composition of per-sample transforms (workers receive it by pickling)."""

    def __init__(self, steps: Sequence[Transform]) -> None:
        self.steps = tuple(steps)

    def __call__(self, sample: dict[str, Any]) -> dict[str, Any]:
        for step in self.steps:
            sample = step(sample)
        return sample


class _WithTransform(Dataset):
    def __init__(self, inner: Dataset, chain: _Chain) -> None:
        self.inner = inner
        self.chain = chain

    def __len__(self) -> int:
        return len(self.inner)  # type: ignore[arg-type]

    def __getitem__(self, i: int) -> dict[str, Any]:
        return self.chain(self.inner[i])


def _one_thread_per_worker(_: int) -> None:
    torch.set_num_threads(1)


@dataclass(frozen=True)
class LoaderPlan:
    """How batches are drawn for one rank of the data-parallel plane."""

    batch_size: int
    rank: int
    world_size: int
    shuffle: bool = True
    num_workers: int = 0
    drop_last: bool = True
    persistent_workers: bool = False
    prefetch_factor: int = 2

    def loader_kwargs(self) -> dict[str, Any]:
        workers = self.num_workers > 0
        kwargs: dict[str, Any] = {"batch_size": self.batch_size, "num_workers": self.num_workers,
                                  "drop_last": self.drop_last, "pin_memory": workers}
        if workers:
            kwargs.update(worker_init_fn=_one_thread_per_worker, persistent_workers=self.persistent_workers,
                          prefetch_factor=self.prefetch_factor)
        return kwargs


class BaseDataset(abc.ABC):
    def __init__(self) -> None:
        self._built: Dataset | None = None
        self._steps: list[Transform] = []

    @abc.abstractmethod
    def build_dataset(self) -> Dataset:
        """The map-style dataset of sample dicts (called once, on first use)."""

    def attach_transform(self, transform: Transform) -> None:
        if self._built is not None:
            raise RuntimeError("the dataset is already built; transforms have to be attached before first use")
        self._steps.append(transform)

    @property
    def transforms(self) -> tuple[Transform, ...]:
        return tuple(self._steps)

    @property
    def dataset(self) -> Dataset:
        if self._built is None:
            raw = self.build_dataset()
            self._built = _WithTransform(raw, _Chain(self._steps)) if self._steps else raw
        return self._built

    @property
    def sample_axes(self) -> str | None:
        """Axis letters of one sample (no batch axis), e.g. "lcxyz"; None when undeclared."""
        return None

    @classmethod
    def resolve_settings(cls, **kwargs: Any) -> dict[str, Any]:
        """The complete settings (after defaults) to record in `resolved_config.json`."""
        return dict(kwargs)

    @classmethod
    def referenced_files(cls, **kwargs: Any) -> tuple[Path, ...]:
        """Files named by the settings, copied into the run directory for provenance."""
        return ()

    def build_dataloader(
        self,
        *,
        batch_size: int,
        rank: int,
        world_size: int,
        shuffle: bool = True,
        num_workers: int = 0,
        drop_last: bool = True,
        persistent_workers: bool = False,
        prefetch_factor: int = 2,
    ) -> DataLoader:
        plan = LoaderPlan(batch_size, rank, world_size, shuffle, num_workers, drop_last, persistent_workers,
                          prefetch_factor)
        sampler = DistributedSampler(self.dataset, num_replicas=plan.world_size, rank=plan.rank, shuffle=plan.shuffle)
        return DataLoader(self.dataset, sampler=sampler, **plan.loader_kwargs())
