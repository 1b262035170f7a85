"""TOML run configuration -> frozen dataclasses (reference `src/utils/config.py:15-154`).

`[model]`, `[algorithm]`, `[data]` and `[val_data]` are registry names plus constructor kwargs;
`[trainer]`, `[parallelism]`, `[init]`, `[augment]` and `[lora]` are strict dataclasses that name any
unknown key. `[lora]` and `[trainer].freeze_backbone_steps` are mutually exclusive: LoRA freezes the
base weights before the optimizer is built, and the unfreeze boundary would then enable gradients
for tensors that no param group holds.
"""

from __future__ import annotations

import dataclasses
import tomllib
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from ..engine.config import AugmentConfig, InitConfig, LoRAConfig, TrainerConfig
from ..parallel.parallel_dims import ParallelDims

COMPONENT_SECTIONS = ("model", "algorithm", "data")


@dataclass(frozen=True)
class ComponentConfig:
    name: str
    kwargs: dict[str, Any] = field(default_factory=dict)


@dataclass(frozen=True)
class RunConfig:
    experiment_name: str
    model: ComponentConfig
    algorithm: ComponentConfig
    data: ComponentConfig
    trainer: TrainerConfig
    parallelism: ParallelDims = field(default_factory=ParallelDims)
    val_data: ComponentConfig | None = None
    init: InitConfig = field(default_factory=InitConfig)
    augment: AugmentConfig = field(default_factory=AugmentConfig)
    lora: LoRAConfig = field(default_factory=LoRAConfig)

    def __post_init__(self) -> None:
        if self.lora.enabled() and self.trainer.freeze_backbone_steps > 0:
            raise ValueError(
                "[lora] and [trainer].freeze_backbone_steps cannot both be set: LoRA keeps the base "
                "weights out of the optimizer, so the unfreeze boundary would allocate gradients "
                "that are never applied. Drop freeze_backbone_steps; a zero-initialised adapter "
                "already starts the encoder at its pretrained function."
            )


def _component(raw: dict[str, Any], section: str) -> ComponentConfig:
    body = dict(raw[section])
    if "name" not in body:
        raise ValueError(f"[{section}] must set 'name' to select a registered implementation")
    return ComponentConfig(name=body.pop("name"), kwargs=body)


def dataclass_from_section(cls: Any, body: dict[str, Any], section: str) -> Any:
    valid = {f.name for f in dataclasses.fields(cls)}
    unknown = sorted(set(body) - valid)
    if unknown:
        raise ValueError(f"[{section}] has unknown key(s) {unknown}; valid keys are {sorted(valid)}")
    return cls(**body)


def parse_run_config(raw: dict[str, Any]) -> RunConfig:
    if "experiment_name" not in raw:
        raise ValueError("config must set a top-level 'experiment_name'")
    missing = [s for s in (*COMPONENT_SECTIONS, "trainer") if s not in raw]
    if missing:
        raise ValueError(f"config is missing required section(s): {missing}")
    return RunConfig(
        experiment_name=raw["experiment_name"],
        model=_component(raw, "model"),
        algorithm=_component(raw, "algorithm"),
        data=_component(raw, "data"),
        trainer=dataclass_from_section(TrainerConfig, dict(raw["trainer"]), "trainer"),
        parallelism=dataclass_from_section(ParallelDims, dict(raw.get("parallelism", {})), "parallelism"),
        val_data=_component(raw, "val_data") if "val_data" in raw else None,
        init=dataclass_from_section(InitConfig, dict(raw.get("init", {})), "init"),
        augment=dataclass_from_section(AugmentConfig, dict(raw.get("augment", {})), "augment"),
        lora=dataclass_from_section(LoRAConfig, dict(raw.get("lora", {})), "lora"),
    )


def load_run_config(path: Path) -> RunConfig:
    with Path(path).open("rb") as handle:
        return parse_run_config(tomllib.load(handle))


def as_plain_dict(config: RunConfig) -> dict[str, Any]:
    return dataclasses.asdict(config)


def flatten_resolved(config: dict[str, Any], prefix: str = "") -> dict[str, Any]:
    """Nested settings as dotted paths. Tuples become lists so a JSON round trip compares equal."""
    flat: dict[str, Any] = {}
    for key, value in config.items():
        path = f"{prefix}{key}"
        if isinstance(value, dict):
            flat.update(flatten_resolved(value, path + "."))
        else:
            flat[path] = list(value) if isinstance(value, tuple) else value
    return flat


def diff_resolved(old: dict[str, Any], new: dict[str, Any]) -> dict[str, tuple[Any, Any]]:
    before, after = flatten_resolved(old), flatten_resolved(new)
    return {
        p: (before.get(p), after.get(p))
        for p in sorted(set(before) | set(after))
        if before.get(p) != after.get(p)
    }
