"""DCP checkpoint save/resume (reference `src/engine/checkpoint.py:25-134`).

Layout: `<run>/checkpoints/step_<N>/` holding `{"model": get_model_state_dict(algorithm),
"optim": get_optimizer_state_dict(...), "train_state": {"step": int64}}`, so keys are the
algorithm's parameter FQNs and a run can resume under a different parallel layout. Planning
collectives go over a Gloo group when the default backend is NCCL (DCP's object collectives are
pickles; only the metadata travels that way, each rank writes its own shards).

Writes are atomic: a step is saved into `step_<N>.tmp` and renamed once every rank has finished,
so a job killed mid-save never leaves a directory that `latest_checkpoint` would pick. Loading
skips (and reports) a step directory without DCP metadata.
"""

from __future__ import annotations

import logging
import shutil
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
import torch.nn as nn
from torch.distributed.checkpoint.state_dict import (
    StateDictOptions,
    get_model_state_dict,
    get_optimizer_state_dict,
    set_model_state_dict,
    set_optimizer_state_dict,
)
from torch.distributed.checkpoint.stateful import Stateful
from torch.optim import Optimizer

logger = logging.getLogger(__name__)

STEP_PREFIX = "step_"
_TMP_SUFFIX = ".tmp"


def coordination_group() -> dist.ProcessGroup | None:
    if not (dist.is_available() and dist.is_initialized()):
        return None
    if dist.get_backend() == "gloo":
        return None
    return dist.new_group(backend="gloo")


class TrainState(Stateful):
    def __init__(self, step: int = 0) -> None:
        self.step = step

    def state_dict(self) -> dict[str, Any]:
        return {"step": torch.tensor(self.step, dtype=torch.int64)}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        self.step = int(state_dict["step"].item())


def _is_complete(path: Path) -> bool:
    return path.is_dir() and not path.name.endswith(_TMP_SUFFIX) and (path / ".metadata").is_file()


def _drop_unsaved_optimizer_state(optim_state: dict[str, Any], path: Path) -> list[str]:
    """A fresh optimizer holds (zero) state for every trainable parameter, a saved one only for the
    parameters that had a gradient by then (an adapter or token that no loss reached yet). Drop the
    entries the checkpoint lacks, so those parameters resume as they were saved: without state."""
    saved = set(dcp.FileSystemReader(str(path)).read_metadata().state_dict_metadata)
    per_param = optim_state.get("state", {})
    unsaved = [fqn for fqn, entry in per_param.items() if any(f"optim.state.{fqn}.{k}" not in saved for k in entry)]
    for fqn in unsaved:
        del per_param[fqn]
    if unsaved:
        logger.warning("checkpoint %s has no optimizer state for %d parameter(s) (no gradient before it was "
                       "saved); they resume without state: %s", path, len(unsaved), ", ".join(unsaved[:8]))
    return unsaved


class CheckpointManager:
    def __init__(self, module: nn.Module, optimizer: Optimizer, checkpoint_dir: Path) -> None:
        self._module = module
        self._optimizer = optimizer
        self._dir = Path(checkpoint_dir)
        self._process_group = coordination_group()

    def _state_dict(self, train_state: TrainState) -> dict[str, Any]:
        return {
            "model": get_model_state_dict(self._module),
            "optim": get_optimizer_state_dict(self._module, self._optimizer),
            "train_state": train_state,
        }

    def _barrier(self) -> None:
        if dist.is_initialized():
            if self._process_group is not None:
                dist.barrier(group=self._process_group)
            else:
                dist.barrier()

    def save(self, step: int) -> Path:
        final = self._dir / f"{STEP_PREFIX}{step}"
        staging = self._dir / f"{STEP_PREFIX}{step}{_TMP_SUFFIX}"
        rank0 = not dist.is_initialized() or dist.get_rank() == 0
        if rank0 and staging.exists():
            shutil.rmtree(staging)
        self._barrier()
        dcp.save(self._state_dict(TrainState(step)), checkpoint_id=str(staging), process_group=self._process_group)
        self._barrier()
        if rank0:
            if final.exists():
                shutil.rmtree(final)
            staging.rename(final)
        self._barrier()
        return final

    def available_steps(self) -> list[int]:
        if not self._dir.is_dir():
            return []
        steps = []
        for p in self._dir.iterdir():
            if p.name.startswith(STEP_PREFIX) and _is_complete(p):
                try:
                    steps.append(int(p.name[len(STEP_PREFIX):]))
                except ValueError:
                    continue
        return sorted(steps)

    def latest_checkpoint(self) -> Path | None:
        steps = self.available_steps()
        return self._dir / f"{STEP_PREFIX}{steps[-1]}" if steps else None

    def load_latest(self) -> int:
        path = self.latest_checkpoint()
        return 0 if path is None else self._load(path)

    def load_step(self, step: int) -> int:
        path = self._dir / f"{STEP_PREFIX}{step}"
        if not _is_complete(path):
            raise ValueError(f"no checkpoint at step {step} in {self._dir}; have {self.available_steps()}")
        return self._load(path)

    def _load(self, path: Path) -> int:
        train_state = TrainState()
        state = self._state_dict(train_state)
        unsaved = _drop_unsaved_optimizer_state(state["optim"], path)
        dcp.load(state, checkpoint_id=str(path), process_group=self._process_group)
        set_model_state_dict(self._module, state["model"])
        set_optimizer_state_dict(self._module, self._optimizer, state["optim"],
                                 options=StateDictOptions(strict=not unsaved))
        return train_state.step
