"""Machine-local settings from `configs/cluster/active.toml` (reference `src/utils/cluster.py:12-46`).

The file is not tracked; `configs/cluster/template.toml` shows its shape. Run artifacts land under
`[environment].checkpoint_dir`, which must be absolute so a job's output does not depend on the
directory it was launched from.
"""

from __future__ import annotations

import tomllib
from pathlib import Path
from typing import Any

REPO_ROOT = Path(__file__).resolve().parents[2]
ACTIVE_CONFIG_PATH = REPO_ROOT / "configs" / "cluster" / "active.toml"
TEMPLATE_CONFIG_PATH = REPO_ROOT / "configs" / "cluster" / "template.toml"


def load_cluster_config(path: Path | None = None) -> dict[str, Any]:
    config_path = path or ACTIVE_CONFIG_PATH
    if not config_path.is_file():
        raise FileNotFoundError(
            f"no cluster configuration at {config_path}; copy {TEMPLATE_CONFIG_PATH} to "
            "active.toml and fill in this machine's paths"
        )
    with config_path.open("rb") as handle:
        return tomllib.load(handle)


def checkpoint_dir(path: Path | None = None) -> Path:
    config_path = path or ACTIVE_CONFIG_PATH
    value = load_cluster_config(config_path).get("environment", {}).get("checkpoint_dir")
    if value is None:
        raise ValueError(f"{config_path} must set [environment].checkpoint_dir")
    resolved = Path(value).expanduser()
    if not resolved.is_absolute():
        raise ValueError(
            f"[environment].checkpoint_dir in {config_path} must be an absolute path; got {value!r}"
        )
    return resolved
