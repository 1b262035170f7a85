"""Dataset contract and dataloader construction (reference `src/data/base.py:11-181`).

A `BaseDataset` builds its torch dataset lazily so transforms can be attached first; attached
transforms compose in attachment order. Loaders shard with `DistributedSampler` over the
data-parallel plane (tensor-parallel peers read the same batch), drop the last partial batch, pin
memory when workers exist, and hold each worker to one intra-op thread so that workers do not
oversubscribe the host that is issuing kernels.
"""

from __future__ import annotations

import abc
from pathlib import Path
from typing import Any

import torch
import torch.utils.data as data


def _single_threaded_worker(worker_id: int) -> None:
    torch.set_num_threads(1)


class TransformedDataset(data.Dataset):
    def __init__(self, source: data.Dataset, transforms: tuple[Any, ...]) -> None:
        self.source = source
        self.transforms = transforms

    def __len__(self) -> int:
        return len(self.source)  # type: ignore[arg-type]

    def __getitem__(self, index: int) -> dict[str, Any]:
        sample = self.source[index]
        for transform in self.transforms:
            sample = transform(sample)
        return sample


class BaseDataset(abc.ABC):
    def __init__(self) -> None:
        self._dataset: data.Dataset | None = None
        self._transforms: tuple[Any, ...] = ()

    @abc.abstractmethod
    def build_dataset(self) -> data.Dataset:
        """Construct the underlying map-style dataset of sample dicts."""

    def attach_transform(self, transform: Any) -> None:
        """Append a per-sample transform; refused once the dataset has been materialised."""
        if self._dataset is not None:
            raise RuntimeError(
                "attach_transform must be called before the dataset is built; samples already "
                "handed out would not see it"
            )
        self._transforms = (*self._transforms, transform)

    @property
    def transforms(self) -> tuple[Any, ...]:
        return self._transforms

    @property
    def dataset(self) -> data.Dataset:
        if self._dataset is None:
            source = self.build_dataset()
            self._dataset = TransformedDataset(source, self._transforms) if self._transforms else source
        return self._dataset

    @property
    def sample_axes(self) -> str | None:
        """Per-sample axis order (batch excluded), e.g. "lcxyz"; None if the data declares none."""
        return None

    @classmethod
    def resolve_settings(cls, **kwargs: Any) -> dict[str, Any]:
        """The dataset's settings fully expanded, for `resolved_config.json`."""
        return dict(kwargs)

    @classmethod
    def referenced_files(cls, **kwargs: Any) -> tuple[Path, ...]:
        """Files the settings point at, copied into the run directory."""
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
    ) -> data.DataLoader:
        sampler = data.DistributedSampler(
            self.dataset, num_replicas=world_size, rank=rank, shuffle=shuffle
        )
        return data.DataLoader(
            self.dataset,
            batch_size=batch_size,
            sampler=sampler,
            num_workers=num_workers,
            drop_last=drop_last,
            pin_memory=num_workers > 0,
            worker_init_fn=_single_threaded_worker if num_workers > 0 else None,
            persistent_workers=persistent_workers and num_workers > 0,
            prefetch_factor=prefetch_factor if num_workers > 0 else None,
        )
