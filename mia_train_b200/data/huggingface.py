"""`hf_semantic_seg`: semantic-segmentation datasets from the HuggingFace Hub
(reference `src/data/huggingface.py:43-312`).

A dataset is a `Preset` (repo, spatial rank, column encoding, image / label / shape columns, the
column naming correlated row groups and how many of its "/"-separated levels form a group, hub
split) or the same fields given inline; any inline field overrides the preset. Encodings:
`"image"` (PNG bytes or decoded images) and `"raw"` (uint8 buffers plus a shape column).

* Splits hold out whole groups (`hold_out_groups`), never rows: `split = "val"` reads exactly the
  held-out groups, `"train"` the rest.
* `row_filters` keeps rows whose column value is in an allowed list.
* Every sample draws a row and a `patch_size` window (zero-padded where the row is smaller) from a
  generator seeded by `(seed, index)`, so samples are reproducible and workers never repeat.
* `samples_per_epoch` fixes the epoch length independently of the row count.
* Samples are `{"img": (1, 1, *patch) float in [0, 1], "label": (1, *patch) int64}` with axes
  `"lcxy"` / `"lcxyz"`; a label id >= `num_classes` is an error.

`datasets` is imported in `build_dataset`, so the registry does not need it.
"""

from __future__ import annotations

import io
from dataclasses import asdict, dataclass
from typing import Any

import numpy as np
import torch
import torch.utils.data as data

from .base import BaseDataset
from .registry import DataRegistry

SAMPLE_AXES = {2: "lcxy", 3: "lcxyz"}


@dataclass(frozen=True)
class Preset:
    repo: str
    spatial_rank: int
    encoding: str
    image_key: str = "image"
    label_key: str = "label"
    shape_key: str | None = None
    group_key: str | None = None
    group_levels: int = 1
    hub_split: str = "train"


def _decode_image(row: dict[str, Any], preset: Preset) -> tuple[np.ndarray, np.ndarray]:
    from PIL import Image

    def load(v: Any) -> np.ndarray:
        if isinstance(v, dict):
            return np.array(Image.open(io.BytesIO(v["bytes"])))
        return np.array(v)

    return load(row[preset.image_key]), load(row[preset.label_key])


def _decode_raw(row: dict[str, Any], preset: Preset) -> tuple[np.ndarray, np.ndarray]:
    if preset.shape_key is None:
        raise ValueError("the 'raw' encoding needs shape_key, the column holding each array's shape")
    shape = tuple(int(s) for s in row[preset.shape_key])
    img = np.frombuffer(row[preset.image_key], dtype=np.uint8).reshape(shape)
    lab = np.frombuffer(row[preset.label_key], dtype=np.uint8).reshape(shape)
    return img, lab


DECODERS = {"image": _decode_image, "raw": _decode_raw}


def group_of(name: str, levels: int) -> str:
    return "/".join(name.split("/")[:levels])


def random_crop(
    image: np.ndarray, label: np.ndarray, size: tuple[int, ...], rng: np.random.Generator
) -> tuple[np.ndarray, np.ndarray]:
    """The same random `size` window of both arrays; short axes are zero-padded at the end."""
    pads, starts = [], []
    for n, want in zip(image.shape, size, strict=True):
        if n < want:
            pads.append((0, want - n))
            starts.append(0)
        else:
            pads.append((0, 0))
            starts.append(int(rng.integers(0, n - want + 1)))
    if any(p != (0, 0) for p in pads):
        image, label = np.pad(image, pads), np.pad(label, pads)
    window = tuple(slice(s, s + w) for s, w in zip(starts, size, strict=True))
    return image[window], label[window]


class _Rows(data.Dataset):
    def __init__(self, rows: Any, owner: HuggingFaceSemanticSegmentation) -> None:
        self.rows = rows
        self.owner = owner

    def __len__(self) -> int:
        return self.owner.samples_per_epoch or len(self.rows)

    def __getitem__(self, index: int) -> dict[str, torch.Tensor]:
        rng = np.random.default_rng((self.owner.seed, index))
        row = self.rows[int(rng.integers(0, len(self.rows)))]
        image, label = DECODERS[self.owner.preset.encoding](row, self.owner.preset)
        image, label = random_crop(image, label, self.owner.patch_size, rng)
        if label.max() >= self.owner.num_classes:
            raise ValueError(f"label id {int(label.max())} >= num_classes={self.owner.num_classes}")
        return {
            "img": torch.from_numpy(np.ascontiguousarray(image)).float().div_(255.0)[None, None],
            "label": torch.from_numpy(np.ascontiguousarray(label)).long()[None],
        }


@DataRegistry.register("hf_semantic_seg")
class HuggingFaceSemanticSegmentation(BaseDataset):
    _PRESET_FIELDS = ("repo", "spatial_rank", "encoding", "image_key", "label_key", "shape_key", "group_key",
                      "group_levels", "hub_split")

    def __init__(
        self,
        patch_size: tuple[int, ...] | list[int],
        preset: str | None = None,
        repo: str | None = None,
        spatial_rank: int | None = None,
        encoding: str | None = None,
        image_key: str | None = None,
        label_key: str | None = None,
        shape_key: str | None = None,
        group_key: str | None = None,
        group_levels: int | None = None,
        hub_split: str | None = None,
        hold_out_groups: tuple[str, ...] | list[str] = (),
        split: str = "train",
        num_classes: int = 64,
        row_filters: dict[str, list[str]] | None = None,
        cache_dir: str | None = None,
        seed: int = 0,
        samples_per_epoch: int | None = None,
    ) -> None:
        super().__init__()
        self.preset = self._resolve_preset(
            preset, repo=repo, spatial_rank=spatial_rank, encoding=encoding, image_key=image_key,
            label_key=label_key, shape_key=shape_key, group_key=group_key, group_levels=group_levels,
            hub_split=hub_split,
        )
        if self.preset.encoding not in DECODERS:
            raise ValueError(f"unknown encoding {self.preset.encoding!r}; expected one of {sorted(DECODERS)}")
        if self.preset.spatial_rank not in SAMPLE_AXES:
            raise ValueError(f"spatial_rank must be 2 or 3, got {self.preset.spatial_rank}")
        if len(patch_size) != self.preset.spatial_rank:
            raise ValueError(
                f"{self.preset.repo} is {self.preset.spatial_rank}-D, so patch_size needs {self.preset.spatial_rank} "
                f"entries, got {list(patch_size)}"
            )
        if split not in ("train", "val"):
            raise ValueError(f"split must be 'train' or 'val', got {split!r}")
        if split == "val" and not hold_out_groups:
            raise ValueError("split='val' needs hold_out_groups: the validation side is exactly the held-out groups")
        if hold_out_groups and self.preset.group_key is None:
            raise ValueError("hold_out_groups needs group_key, the column to split on")
        self.patch_size = tuple(int(p) for p in patch_size)
        self.hold_out_groups = tuple(hold_out_groups)
        self.split = split
        self.num_classes = int(num_classes)
        self.row_filters = dict(row_filters or {})
        self.cache_dir = cache_dir
        self.seed = int(seed)
        self.samples_per_epoch = samples_per_epoch

    @staticmethod
    def _resolve_preset(name: str | None, **fields: Any) -> Preset:
        given = {k: v for k, v in fields.items() if v is not None}
        if name is not None:
            if name not in PRESETS:
                raise ValueError(f"unknown preset {name!r}; expected one of {sorted(PRESETS)}")
            return Preset(**{**asdict(PRESETS[name]), **given})
        missing = [k for k in ("repo", "spatial_rank", "encoding") if k not in given]
        if missing:
            raise ValueError(f"without a preset, {missing} must be given; presets: {sorted(PRESETS)}")
        return Preset(**given)

    def select_rows(self, rows: Any) -> Any:
        """Apply row filters and the group hold-out to a `datasets.Dataset`-like table."""
        for column, allowed in self.row_filters.items():
            if column not in rows.column_names:
                raise ValueError(
                    f"row_filters names column {column!r}, which {self.preset.repo} lacks; columns: {rows.column_names}"
                )
            values = rows[column]
            rows = rows.select([i for i, v in enumerate(values) if v in allowed])
        if self.preset.group_key is not None:
            held = set(self.hold_out_groups)
            groups = [group_of(n, self.preset.group_levels) for n in rows[self.preset.group_key]]
            val = self.split == "val"
            keep = [i for i, g in enumerate(groups) if (g in held) == val]
            if not keep:
                raise ValueError(
                    f"no rows left for split={self.split!r} after holding out {sorted(held)}; groups present: "
                    f"{sorted(set(groups))}"
                )
            rows = rows.select(keep)
        if len(rows) == 0:
            raise ValueError(f"{self.preset.repo} yielded no rows after filtering")
        return rows

    def build_dataset(self) -> data.Dataset:
        try:
            import datasets
        except ImportError as error:
            raise ImportError("hf_semantic_seg reads the Hub through the `datasets` package, which is missing") from error
        rows = datasets.load_dataset(self.preset.repo, split=self.preset.hub_split, cache_dir=self.cache_dir)
        return _Rows(self.select_rows(rows), self)

    @property
    def sample_axes(self) -> str:
        return SAMPLE_AXES[self.preset.spatial_rank]

    @classmethod
    def resolve_settings(cls, **kwargs: Any) -> dict[str, Any]:
        preset = cls._resolve_preset(kwargs.get("preset"), **{k: kwargs.get(k) for k in cls._PRESET_FIELDS})
        return {**kwargs, **asdict(preset)}


PRESETS: dict[str, Preset] = {
    "cellmap_3d": Preset(repo="eminorhan/cellmap-3d", spatial_rank=3, encoding="raw", image_key="volume",
                         shape_key="shape", group_key="crop_name"),
    "cellmap_2d": Preset(repo="eminorhan/cellmap-2d", spatial_rank=2, encoding="image", group_key="crop_name"),
}
