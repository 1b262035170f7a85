"""Run orchestration: config -> process group -> mesh -> run directory -> trainer -> train.

Follows the reference's `src/engine/run.py:32-348`: rank 0 picks (or, with `--resume`, finds) the
`<experiment>_<YYYYmmdd_HHMMSS>` directory and broadcasts it; rank 0 writes the provenance files
and checks a resumed run's settings (refusing changes under `model.`, `algorithm.name` or
`lora.`), and broadcasts success or the error so every rank raises together instead of hanging in
the barrier; the model is built, LoRA-adapted and then initialised from `[init]` (in that order);
the algorithm is built around the model and the training dataset.
"""

from __future__ import annotations

import dataclasses
import json
from datetime import datetime
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from ..algorithms.registry import AlgorithmRegistry
from ..data.augment import VolumeAugmentation
from ..data.registry import DataRegistry
from ..models.registry import ModelRegistry
from ..parallel.setup import destroy_distributed, device_type, init_distributed
from ..utils.cluster import REPO_ROOT, checkpoint_dir
from ..utils.config import RunConfig, as_plain_dict, diff_resolved, load_run_config
from ..utils.pretrained import load_pretrained
from ..utils.provenance import write_run_artifacts
from .lora import apply_lora
from .trainer import Trainer

RESUME_LATEST = "latest"
INCOMPATIBLE_ON_RESUME = ("model.", "algorithm.name", "lora.")


def latest_run_dir(output_root: Path, experiment_name: str) -> Path | None:
    if not output_root.is_dir():
        return None
    prefix = f"{experiment_name}_"
    runs = sorted(p for p in output_root.iterdir() if p.is_dir() and p.name.startswith(prefix))
    return runs[-1] if runs else None


def resolve_output_dir(output_root: Path, experiment_name: str, resume: str | None = None) -> Path:
    if resume is not None and resume != RESUME_LATEST:
        chosen = Path(resume)
        if not chosen.is_dir():
            raise ValueError(
                f"--resume {resume!r} is not an existing directory; omit --resume for a fresh run or "
                f"pass --resume {RESUME_LATEST} to continue the most recent one"
            )
        return chosen
    name = [""]
    if not dist.is_initialized() or dist.get_rank() == 0:
        existing = latest_run_dir(output_root, experiment_name) if resume else None
        name[0] = existing.name if existing else f"{experiment_name}_{datetime.now().strftime('%Y%m%d_%H%M%S')}"
    if dist.is_initialized():
        dist.broadcast_object_list(name, src=0)
    return output_root / name[0]


def report_resumed_config(output_dir: Path, resolved: dict[str, Any]) -> None:
    stored_path = output_dir / "resolved_config.json"
    if not stored_path.is_file():
        return
    changes = diff_resolved(json.loads(stored_path.read_text(encoding="utf-8")), resolved)
    if not changes:
        return
    bad = {p: c for p, c in changes.items() if any(p.startswith(x) for x in INCOMPATIBLE_ON_RESUME)}
    if bad:
        detail = "; ".join(f"{p}: {o!r} -> {n!r}" for p, (o, n) in bad.items())
        raise ValueError(
            f"cannot resume {output_dir.name}: the architecture changed since it was started ({detail}); "
            "start a fresh run under a new experiment_name instead"
        )
    detail = "; ".join(f"{p}: {o!r} -> {n!r}" for p, (o, n) in changes.items())
    print(f"[resume] continuing {output_dir.name} with changed settings: {detail}", flush=True)


def resolved_settings(config: RunConfig) -> dict[str, Any]:
    resolved = as_plain_dict(config)
    for section in ("data", "val_data"):
        comp = getattr(config, section)
        if comp is not None:
            resolved[section]["kwargs"] = DataRegistry.get(comp.name).resolve_settings(**comp.kwargs)
    return resolved


def referenced_config_files(config: RunConfig) -> tuple[Path, ...]:
    seen: dict[Path, None] = {}
    for section in ("data", "val_data"):
        comp = getattr(config, section)
        if comp is not None:
            for path in DataRegistry.get(comp.name).referenced_files(**comp.kwargs):
                seen[Path(path)] = None
    return tuple(seen)


def prepare_run_dir(
    output_dir: Path, config_path: Path, resolved: dict[str, Any], rank: int, referenced: tuple[Path, ...] = ()
) -> None:
    failure: list[str | None] = [None]
    if rank == 0:
        try:
            report_resumed_config(output_dir, resolved)
            write_run_artifacts(output_dir, config_path, resolved, REPO_ROOT, referenced)
        except Exception as error:  # noqa: BLE001 - forwarded to every rank
            failure[0] = f"{type(error).__name__}: {error}"
    if dist.is_initialized():
        dist.broadcast_object_list(failure, src=0)
    if failure[0] is not None:
        raise RuntimeError(f"could not prepare {output_dir}: {failure[0]}")
    if dist.is_initialized():
        dist.barrier()


def _init_kwargs(config: RunConfig) -> dict[str, Any]:
    i = config.init
    return {
        "prefix": i.prefix,
        "inflate": i.inflate_2d_to_3d,
        "skip": i.skip,
        "strict": i.strict,
        "allow_unused": i.allow_unused,
        "merge_lora": i.merge_lora,
    }


def prepare_model(config: RunConfig) -> Any:
    """Build the model, then LoRA, then `[init]` (adapter tensors in a checkpoint need a home)."""
    model = ModelRegistry.build(config.model.name, **config.model.kwargs)
    if config.lora.enabled():
        print(f"[lora] {apply_lora(model, config.lora).summary()}", flush=True)
    if config.init.path and config.init.target == "model":
        load_pretrained(model, config.init.path, **_init_kwargs(config))
    return model


def build_trainer(
    config: RunConfig, output_dir: Path, mesh: DeviceMesh | None = None, device: torch.device | None = None
) -> Trainer:
    train_dataset = DataRegistry.build(config.data.name, **config.data.kwargs)
    if config.augment.enabled():
        train_dataset.attach_transform(
            VolumeAugmentation(sample_axes=train_dataset.sample_axes, **dataclasses.asdict(config.augment))
        )
        print(f"[augment] training data: {config.augment}", flush=True)
    val_dataset = DataRegistry.build(config.val_data.name, **config.val_data.kwargs) if config.val_data else None
    model = prepare_model(config)
    algorithm = AlgorithmRegistry.build(config.algorithm.name, model, train_dataset, **config.algorithm.kwargs)
    if config.init.path and config.init.target == "algorithm":
        load_pretrained(algorithm, config.init.path, **_init_kwargs(config))
    transform = algorithm.sample_transform()
    if transform is not None:
        for ds in (train_dataset, val_dataset):
            if ds is not None:
                ds.attach_transform(transform)
        print(f"[data] {type(transform).__name__} runs in the dataloader workers", flush=True)
    return Trainer(
        algorithm=algorithm,
        train_dataset=train_dataset,
        config=config.trainer,
        output_dir=output_dir,
        dims=config.parallelism,
        mesh=mesh,
        val_dataset=val_dataset,
        device=device,
    )


def run(config_path: Path, output_root: Path | None = None, resume: str | None = None) -> Path:
    from .. import components  # noqa: F401  (populates the registries the config names)

    config = load_run_config(Path(config_path))
    root = Path(output_root) if output_root is not None else checkpoint_dir()
    rank, _, local_rank = init_distributed()
    try:
        mesh = config.parallelism.build_mesh(device_type())
        device = torch.device("cuda", local_rank) if torch.cuda.is_available() else torch.device("cpu")
        output_dir = resolve_output_dir(root, config.experiment_name, resume)
        prepare_run_dir(output_dir, Path(config_path), resolved_settings(config), rank, referenced_config_files(config))
        build_trainer(config, output_dir, mesh=mesh, device=device).train()
    finally:
        destroy_distributed()
    return output_dir
