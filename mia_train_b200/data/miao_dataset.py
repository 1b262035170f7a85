"""`miao_volumes`: multi-scale OME-NGFF patches read by the external `miao` package
(reference `src/data/miao_dataset.py:20-118`).

Every `[data]` key except `name` and `config_path` is a `miao.MiaoConfig` field. `config_path`
names a miao YAML that is loaded first (relative paths resolve against the repository root, not
the working directory); inline keys override it. Unknown keys are rejected (miao's config would
otherwise ignore a misspelling). `resolve_settings` expands the merged configuration into plain
values for the run record, and `referenced_files` reports the YAML so the run directory keeps a
copy. `sample_axes` is miao's `output_axes` (it must contain "l").

`miao` is imported when the dataset is used, not when it is registered, so configs that do not
name this dataset run without it.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

import torch.utils.data as data

from .base import BaseDataset
from .registry import DataRegistry

_REPO_ROOT = Path(__file__).resolve().parents[2]


def _miao() -> tuple[Any, Any, Any]:
    try:
        from miao.config import MiaoConfig, load_config
        from miao.dataset import VolumeDataset
    except ImportError as error:
        raise ImportError(
            "the miao_volumes dataset reads OME-NGFF volumes through the `miao` package, which is not "
            "installed; install it, or use the synthetic_volumes / hf_semantic_seg datasets"
        ) from error
    return MiaoConfig, load_config, VolumeDataset


@DataRegistry.register("miao_volumes")
class MiaoVolumeDataset(BaseDataset):
    def __init__(self, config_path: str | Path | None = None, **miao_config: Any) -> None:
        super().__init__()
        config_cls, _, _ = _miao()
        self.config = config_cls(**self.resolve_settings(config_path=config_path, **miao_config))

    @classmethod
    def resolve_settings(cls, config_path: str | Path | None = None, **miao_config: Any) -> dict[str, Any]:
        config_cls, _, _ = _miao()
        fields = set(config_cls.model_fields)
        unknown = sorted(set(miao_config) - fields)
        if unknown:
            raise ValueError(
                f"unknown [data] key(s) for miao_volumes: {unknown}; valid keys are {sorted(fields)} "
                "(plus 'config_path')"
            )
        merged: dict[str, Any] = {}
        if config_path is not None:
            merged.update(cls._from_yaml(config_path))
        merged.update(miao_config)
        return config_cls(**merged).model_dump(mode="json")

    @classmethod
    def referenced_files(cls, config_path: str | Path | None = None, **miao_config: Any) -> tuple[Path, ...]:
        return () if config_path is None else (cls._resolve_path(config_path),)

    @staticmethod
    def _resolve_path(config_path: str | Path) -> Path:
        path = Path(config_path)
        if not path.is_absolute():
            path = _REPO_ROOT / path
        if not path.is_file():
            raise FileNotFoundError(
                f"[data] config_path={str(config_path)!r} does not exist (looked at {path}); relative paths "
                "resolve against the repository root"
            )
        return path

    @classmethod
    def _from_yaml(cls, config_path: str | Path) -> dict[str, Any]:
        _, load_config, _ = _miao()
        return load_config(cls._resolve_path(config_path)).model_dump()

    @property
    def sample_axes(self) -> str | None:
        return str(self.config.output_axes)

    def build_dataset(self) -> data.Dataset:
        _, _, volume_dataset = _miao()
        return volume_dataset(self.config)
