"""What a run directory records about how each attempt was started.

Interface of reference `src/utils/provenance.py:28-107`: the file names below are what tooling and
people look for in a run directory, so they are kept; the code is this framework's own.

* `config.<ext>`         the TOML the run was launched with (overwritten on resume)
* `<name>`               copies of files the config points at (data configs), same base name
* `resolved_config.json` every setting after defaults were filled in
* `git_commit.txt`       the source revision, suffixed `(dirty)` when the tree had changes
* `dirty.patch`          those changes, against HEAD
* `attempts.log`         one appended line per launch or resume, so the history survives resumes
"""

from __future__ import annotations

import json
import shutil
import subprocess
from collections.abc import Sequence
from dataclasses import dataclass
from datetime import datetime
from pathlib import Path
from typing import Any


@dataclass(frozen=True)
class SourceState:
    """The repository revision a run was started from (None fields: not a git checkout)."""

    commit: str | None
    patch: str = ""

    @property
    def dirty(self) -> bool:
        return bool(self.patch.strip())

    def describe(self) -> str:
        if self.commit is None:
            return "unknown"
        return f"{self.commit} (dirty)" if self.dirty else self.commit

    @classmethod
    def probe(cls, repo_dir: Path) -> SourceState:
        def ask(*args: str) -> str | None:
            try:
                done = subprocess.run(["git", "-C", str(repo_dir), *args], capture_output=True, text=True)
            except OSError:  # no git binary
                return None
            return done.stdout if done.returncode == 0 else None

        head = ask("rev-parse", "--verify", "HEAD")
        if head is None:
            return cls(None)
        return cls(head.strip(), ask("diff", "HEAD") or "")


def _gather_copies(config_path: Path, referenced: Sequence[Path]) -> dict[str, Path]:
    """Destination name -> source; two different sources may not share a name."""
    plan: dict[str, Path] = {"config" + config_path.suffix: config_path}
    for src in referenced:
        other = plan.get(src.name)
        if other is not None and other.resolve() != src.resolve():
            raise ValueError(
                f"cannot record both {other} and {src} in the run directory: they share the file name "
                f"{src.name!r}; give one of them another name"
            )
        plan[src.name] = src
    return plan


def write_run_artifacts(
    output_dir: Path,
    config_path: Path,
    resolved_config: dict[str, Any],
    repo_dir: Path,
    referenced_files: Sequence[Path] = (),
) -> None:
    """Record this attempt in `output_dir` (created if needed)."""
    output_dir = Path(output_dir)
    copies = _gather_copies(Path(config_path), [Path(p) for p in referenced_files])
    output_dir.mkdir(parents=True, exist_ok=True)
    for dest, src in copies.items():
        shutil.copyfile(src, output_dir / dest)
    (output_dir / "resolved_config.json").write_text(
        json.dumps(resolved_config, indent=2, sort_keys=False, default=str), encoding="utf-8"
    )
    state = SourceState.probe(Path(repo_dir))
    if state.commit is None:
        revision = f"unavailable: {repo_dir} is not a git checkout, so no source revision was recorded"
    else:
        revision = state.describe()
        if state.dirty:
            (output_dir / "dirty.patch").write_text(state.patch, encoding="utf-8")
    (output_dir / "git_commit.txt").write_text(revision + "\n", encoding="utf-8")
    stamp = datetime.now().isoformat(timespec="seconds")
    with open(output_dir / "attempts.log", "a", encoding="utf-8") as log:
        log.write(f"{stamp}  {state.describe() if state.commit else 'no git checkout'}\n")
