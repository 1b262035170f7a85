"""Run-directory provenance (reference `src/utils/provenance.py:28-107`).

Every attempt records the source config, the fully resolved settings as JSON, the git commit (with
`(dirty)` and a `dirty.patch` when the tree has local changes), copies of referenced data configs,
and one line in `attempts.log`, which survives resumes that overwrite the other files.
"""

from __future__ import annotations

import json
import shutil
import subprocess
from collections.abc import Sequence
from datetime import datetime
from pathlib import Path
from typing import Any


def _git(repo_dir: Path, *args: str) -> str | None:
    try:
        result = subprocess.run(
            ["git", "-C", str(repo_dir), *args], capture_output=True, text=True, check=False
        )
    except OSError:
        return None
    return result.stdout if result.returncode == 0 else None


def git_metadata(repo_dir: Path) -> dict[str, Any] | None:
    commit = _git(repo_dir, "rev-parse", "HEAD")
    if commit is None:
        return None
    diff = _git(repo_dir, "diff", "HEAD") or ""
    return {"commit": commit.strip(), "dirty": bool(diff.strip()), "diff": diff}


def write_run_artifacts(
    output_dir: Path,
    config_path: Path,
    resolved_config: dict[str, Any],
    repo_dir: Path,
    referenced_files: Sequence[Path] = (),
) -> None:
    output_dir.mkdir(parents=True, exist_ok=True)
    shutil.copyfile(config_path, output_dir / f"config{config_path.suffix}")
    _copy_referenced(output_dir, config_path, referenced_files)
    (output_dir / "resolved_config.json").write_text(
        json.dumps(resolved_config, indent=2, default=str), encoding="utf-8"
    )
    meta = git_metadata(repo_dir)
    if meta is None:
        (output_dir / "git_commit.txt").write_text(
            f"no git repository at {repo_dir}; run provenance unavailable\n", encoding="utf-8"
        )
        _append_attempt(output_dir, "no git repository")
        return
    stamp = meta["commit"] + (" (dirty)" if meta["dirty"] else "")
    (output_dir / "git_commit.txt").write_text(stamp + "\n", encoding="utf-8")
    if meta["dirty"]:
        (output_dir / "dirty.patch").write_text(meta["diff"], encoding="utf-8")
    _append_attempt(output_dir, stamp)


def _copy_referenced(output_dir: Path, config_path: Path, files: Sequence[Path]) -> None:
    taken: dict[str, Path] = {f"config{config_path.suffix}": config_path}
    for source in files:
        clash = taken.get(source.name)
        if clash is not None and clash.resolve() != source.resolve():
            raise ValueError(
                f"two different config files are both named {source.name!r} ({clash} and {source}); "
                "rename one so the run directory can keep both"
            )
        taken[source.name] = source
        shutil.copyfile(source, output_dir / source.name)


def _append_attempt(output_dir: Path, stamp: str) -> None:
    with (output_dir / "attempts.log").open("a", encoding="utf-8") as handle:
        handle.write(f"{datetime.now().isoformat(timespec='seconds')}  {stamp}\n")
