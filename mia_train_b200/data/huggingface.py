"""`hf_semantic_seg`: 2-D / 3-D semantic-segmentation crops read from HuggingFace Hub tables.

Config interface of reference `src/data/huggingface.py:43-312` (keys, preset names and the public
Hub repositories and columns they point at); the implementation is this framework's own.

A table is described by a `Preset`: repository, spatial rank, how images are stored
(`"image"`: PNG bytes or decoded images; `"raw"`: uint8 buffers next to a shape column), the
image / label / shape columns, a group column whose first `group_levels` "/"-separated parts name
a group of correlated rows, and the Hub split to read. Inline keys override a named preset.

Row selection is one pass that computes a keep-mask: `row_filters` (column -> allowed values)
and the group hold-out (`split = "val"` keeps exactly the rows of `hold_out_groups`, `"train"` the
others), so no group ever appears on both sides. Each sample index seeds its own generator with
`(seed, index)`, picks a row and a `patch_size` window from it (axes shorter than the window are
zero-filled past their end) -- reproducible, and different in every worker. `samples_per_epoch`
fixes the epoch length whatever the number of rows. Samples are `{"img": (1, 1, *patch) float in
[0, 1], "label": (1, *patch) int64}` with axes `"lcxy"` / `"lcxyz"`; a label id beyond
`num_classes - 1` raises. The `datasets` package is imported only when the table is first read.
"""

from __future__ import annotations

import dataclasses
import io
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch
from torch.utils.data import Dataset

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


PRESETS: dict[str, Preset] = {
    "cellmap_3d": Preset(repo="eminorhan/cellmap-3d", spatial_rank=3, encoding="raw", image_key="volume",
                         shape_key="shape", group_key="crop_name"),
    "cellmap_2d": Preset(repo="eminorhan/cellmap-2d", spatial_rank=2, encoding="image", group_key="crop_name"),
}
_PRESET_FIELDS = tuple(f.name for f in dataclasses.fields(Preset))
ENCODINGS = ("image", "raw")


def group_of(name: str, levels: int) -> str:
    """The group a row belongs to: the first `levels` parts of its "/"-separated name."""
    parts = name.split("/")
    return "/".join(parts[: max(1, levels)])


def random_crop(image: np.ndarray, label: np.ndarray, size: tuple[int, ...],
                rng: np.random.Generator) -> tuple[np.ndarray, np.ndarray]:
    """The same window of `size` from both arrays, at a random start; where an axis is shorter than
    the window, the window starts at 0 and the part past the array's end is zero."""
    starts = [int(rng.integers(0, n - w + 1)) if n >= w else 0 for n, w in zip(image.shape, size, strict=True)]
    src = tuple(slice(s, s + min(w, n)) for s, w, n in zip(starts, size, image.shape, strict=True))
    dst = tuple(slice(0, min(w, n)) for w, n in zip(size, image.shape, strict=True))
    out_img = np.zeros(size, dtype=image.dtype)
    out_lab = np.zeros(size, dtype=label.dtype)
    out_img[dst] = image[src]
    out_lab[dst] = label[src]
    return out_img, out_lab


def _decode(row: dict[str, Any], layout: Preset) -> tuple[np.ndarray, np.ndarray]:
    """(image, label) arrays of one table row."""
    if layout.encoding == "raw":
        if layout.shape_key is None:
            raise ValueError("raw-encoded tables need shape_key (the column with each array's shape)")
        shape = [int(n) for n in row[layout.shape_key]]
        return tuple(np.frombuffer(row[k], dtype=np.uint8).reshape(shape)  # type: ignore[return-value]
                     for k in (layout.image_key, layout.label_key))
    from PIL import Image

    def as_array(cell: Any) -> np.ndarray:
        if isinstance(cell, dict) and "bytes" in cell:
            cell = Image.open(io.BytesIO(cell["bytes"]))
        return np.asarray(cell)

    return as_array(row[layout.image_key]), as_array(row[layout.label_key])


class _Crops(Dataset):
    def __init__(self, rows: Any, source: HuggingFaceSemanticSegmentation) -> None:
        self.rows = rows
        self.layout = source.preset
        self.patch = source.patch_size
        self.classes = source.num_classes
        self.seed = source.seed
        self.length = source.samples_per_epoch or len(rows)

    def __len__(self) -> int:
        return self.length

    def __getitem__(self, index: int) -> dict[str, torch.Tensor]:
        rng = np.random.default_rng([self.seed, index])
        image, label = _decode(self.rows[int(rng.integers(len(self.rows)))], self.layout)
        image, label = random_crop(image, label, self.patch, rng)
        top = int(label.max(initial=0))
        if top >= self.classes:
            raise ValueError(f"a label holds class id {top}, but num_classes = {self.classes}")
        img = torch.as_tensor(np.ascontiguousarray(image), dtype=torch.float32) / 255.0
        return {"img": img.reshape(1, 1, *self.patch), "label": torch.as_tensor(label.astype(np.int64))[None]}


@DataRegistry.register("hf_semantic_seg")
class HuggingFaceSemanticSegmentation(BaseDataset):
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
        overrides = dict(repo=repo, spatial_rank=spatial_rank, encoding=encoding, image_key=image_key,
                         label_key=label_key, shape_key=shape_key, group_key=group_key, group_levels=group_levels,
                         hub_split=hub_split)
        self.preset = self._resolve_preset(preset, **overrides)
        layout = self.preset
        problems = []
        if layout.encoding not in ENCODINGS:
            problems.append(f"encoding {layout.encoding!r} is not one of {', '.join(ENCODINGS)}")
        if layout.spatial_rank not in SAMPLE_AXES:
            problems.append(f"spatial_rank {layout.spatial_rank} is not 2 or 3")
        elif len(patch_size) != layout.spatial_rank:
            problems.append(f"patch_size {list(patch_size)} needs {layout.spatial_rank} entries for {layout.repo}")
        if split not in ("train", "val"):
            problems.append(f"split {split!r} is neither 'train' nor 'val'")
        if split == "val" and not hold_out_groups:
            problems.append("split = 'val' reads the held-out groups, so hold_out_groups cannot be empty")
        if hold_out_groups and layout.group_key is None:
            problems.append("hold_out_groups needs a group_key column to decide group membership")
        if problems:
            raise ValueError("hf_semantic_seg: " + "; ".join(problems))
        self.patch_size = tuple(int(p) for p in patch_size)
        self.hold_out_groups = tuple(hold_out_groups)
        self.split = split
        self.num_classes = int(num_classes)
        self.row_filters = {k: list(v) for k, v in (row_filters or {}).items()}
        self.cache_dir = cache_dir
        self.seed = int(seed)
        self.samples_per_epoch = samples_per_epoch

    @staticmethod
    def _resolve_preset(name: str | None, **fields: Any) -> Preset:
        given = {k: v for k, v in fields.items() if v is not None}
        if name is None:
            needed = [k for k in ("repo", "spatial_rank", "encoding") if k not in given]
            if needed:
                raise ValueError(f"hf_semantic_seg: name a preset ({', '.join(sorted(PRESETS))}) or give "
                                 f"{', '.join(needed)}")
            return Preset(**given)
        if name not in PRESETS:
            raise ValueError(f"hf_semantic_seg: preset {name!r} is unknown (known: {', '.join(sorted(PRESETS))})")
        return dataclasses.replace(PRESETS[name], **given)

    def select_rows(self, rows: Any) -> Any:
        """The rows of this split that pass the filters (`rows` is a `datasets.Dataset`-like table)."""
        n = len(rows)
        keep = np.ones(n, dtype=bool)
        for column, allowed in self.row_filters.items():
            if column not in rows.column_names:
                raise ValueError(f"row_filters: {self.preset.repo} has no column {column!r} "
                                 f"(columns: {', '.join(rows.column_names)})")
            accepted = set(allowed)
            keep &= np.fromiter((v in accepted for v in rows[column]), dtype=bool, count=n)
        if self.preset.group_key is not None:
            held = set(self.hold_out_groups)
            names = rows[self.preset.group_key]
            in_held = np.fromiter((group_of(v, self.preset.group_levels) in held for v in names), dtype=bool, count=n)
            keep &= in_held if self.split == "val" else ~in_held
        chosen = np.flatnonzero(keep).tolist()
        if not chosen:
            raise ValueError(f"hf_semantic_seg: no rows of {self.preset.repo} remain for split {self.split!r} "
                             f"(held-out groups {sorted(self.hold_out_groups)}, filters {self.row_filters})")
        return rows.select(chosen)

    def build_dataset(self) -> Dataset:
        try:
            import datasets
        except ImportError as error:
            raise ImportError("hf_semantic_seg needs the `datasets` package to read Hub tables") from error
        table = datasets.load_dataset(self.preset.repo, split=self.preset.hub_split, cache_dir=self.cache_dir)
        return _Crops(self.select_rows(table), self)

    @property
    def sample_axes(self) -> str:
        return SAMPLE_AXES[self.preset.spatial_rank]

    @classmethod
    def resolve_settings(cls, **kwargs: Any) -> dict[str, Any]:
        layout = cls._resolve_preset(kwargs.get("preset"), **{k: kwargs.get(k) for k in _PRESET_FIELDS})
        return {**kwargs, **dataclasses.asdict(layout)}
