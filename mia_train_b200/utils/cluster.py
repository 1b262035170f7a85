"""Per-machine settings (interface of reference `src/utils/cluster.py:12-46`).

A machine keeps its own paths in `configs/cluster/active.toml` (untracked; the tracked
`template.toml` documents the keys). The framework reads exactly one of them at run time: the root
under which run directories are created, `[environment].checkpoint_dir`. Relative roots are refused
because a resubmitted job may start in another working directory and must find the same runs.
"""

from __future__ import annotations

import tomllib
from dataclasses import dataclass
from pathlib import Path
from typing import Any

REPO_ROOT = Path(__file__).resolve().parents[2]
CLUSTER_DIR = REPO_ROOT / "configs" / "cluster"
ACTIVE_CONFIG_PATH = CLUSTER_DIR / "active.toml"
TEMPLATE_CONFIG_PATH = CLUSTER_DIR / "template.toml"


@dataclass(frozen=True)
class ClusterSettings:
    """The parsed machine file and where it came from."""

    source: Path
    tables: dict[str, Any]

    @classmethod
    def read(cls, path: Path | None = None) -> ClusterSettings:
        source = Path(path) if path is not None else ACTIVE_CONFIG_PATH
        try:
            raw = source.read_bytes()
        except FileNotFoundError:
            raise FileNotFoundError(
                f"machine settings file {source} is missing: start from {TEMPLATE_CONFIG_PATH} "
                "(save it as active.toml next to it) and set the paths of this machine"
            ) from None
        return cls(source, tomllib.loads(raw.decode("utf-8")))

    def get(self, table: str, key: str) -> Any:
        return self.tables.get(table, {}).get(key)

    @property
    def checkpoint_root(self) -> Path:
        value = self.get("environment", "checkpoint_dir")
        if value is None:
            raise ValueError(f"{self.source}: the [environment] table needs a checkpoint_dir entry")
        root = Path(str(value)).expanduser()
        if not root.is_absolute():
            raise ValueError(
                f"{self.source}: checkpoint_dir = {value!r} is relative; runs are located from it on "
                "every (re)submission, so give an absolute path"
            )
        return root


def load_cluster_config(path: Path | None = None) -> dict[str, Any]:
    """All tables of the machine file (raises FileNotFoundError with a hint when it is absent)."""
    return ClusterSettings.read(path).tables


def checkpoint_dir(path: Path | None = None) -> Path:
    """The absolute root for run directories, from `[environment].checkpoint_dir`."""
    return ClusterSettings.read(path).checkpoint_root
