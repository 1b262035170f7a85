"""Run configuration: one TOML file, parsed into frozen dataclasses.

The section and key names are the reference's contract (`src/utils/config.py:15-154`), so a config
written for it loads here unchanged:

* component sections `[model]`, `[algorithm]`, `[data]` (required) and `[val_data]` (optional):
  `name` picks a registered implementation, every other key goes to its constructor;
* settings sections `[trainer]` (required), `[parallelism]`, `[init]`, `[augment]`, `[lora]`: keys
  must be fields of the section's dataclass, and an unknown key is an error naming the valid ones;
* a top-level `experiment_name`.

The parser is driven by the `_SECTIONS` table below. One rule spans sections: `[lora]` and
`[trainer].freeze_backbone_steps` exclude each other (LoRA leaves the base weights out of the
optimizer before it is built; the unfreeze step would then create gradients nobody applies).
"""

from __future__ import annotations

import dataclasses
import tomllib
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from ..engine.config import AugmentConfig, InitConfig, LoRAConfig, TrainerConfig
from ..parallel.parallel_dims import ParallelDims


@dataclass(frozen=True)
class ComponentConfig:
    """A registry name and the constructor keyword arguments that go with it."""

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
                "a [lora] adapter cannot be combined with [trainer].freeze_backbone_steps: the base "
                "weights are outside the optimizer, so unfreezing them would only add unused gradients "
                "(a zero-initialised adapter already starts from the pretrained encoder; remove "
                "freeze_backbone_steps)"
            )


# section -> (dataclass, or None for a component section; required)
_SECTIONS: dict[str, tuple[type | None, bool]] = {
    "model": (None, True),
    "algorithm": (None, True),
    "data": (None, True),
    "val_data": (None, False),
    "trainer": (TrainerConfig, True),
    "parallelism": (ParallelDims, False),
    "init": (InitConfig, False),
    "augment": (AugmentConfig, False),
    "lora": (LoRAConfig, False),
}


def _component(section: str, table: dict[str, Any]) -> ComponentConfig:
    kwargs = {k: v for k, v in table.items() if k != "name"}
    if "name" not in table:
        raise ValueError(f"[{section}] needs a 'name' key selecting one of the registered implementations")
    return ComponentConfig(str(table["name"]), kwargs)


def _settings(section: str, cls: type, table: dict[str, Any]) -> Any:
    allowed = [f.name for f in dataclasses.fields(cls)]
    stray = sorted(k for k in table if k not in allowed)
    if stray:
        raise ValueError(f"[{section}]: unknown key(s) {', '.join(stray)} (accepted keys: {', '.join(sorted(allowed))})")
    return cls(**table)


def parse_run_config(raw: dict[str, Any]) -> RunConfig:
    """Build a `RunConfig` from an already-parsed TOML document."""
    if "experiment_name" not in raw:
        raise ValueError("the config has no top-level experiment_name")
    absent = [name for name, (_, required) in _SECTIONS.items() if required and name not in raw]
    if absent:
        raise ValueError(f"the config is missing the required section(s) {', '.join(absent)}")
    parsed: dict[str, Any] = {}
    for name, (cls, _) in _SECTIONS.items():
        if name not in raw:
            continue
        table = dict(raw[name])
        parsed[name] = _component(name, table) if cls is None else _settings(name, cls, table)
    return RunConfig(experiment_name=raw["experiment_name"], **parsed)


def load_run_config(path: Path) -> RunConfig:
    return parse_run_config(tomllib.loads(Path(path).read_text(encoding="utf-8")))


def as_plain_dict(config: RunConfig) -> dict[str, Any]:
    """Every resolved setting as nested plain containers (what `resolved_config.json` stores)."""
    return dataclasses.asdict(config)


def flatten_resolved(config: dict[str, Any], prefix: str = "") -> dict[str, Any]:
    """{"a": {"b": 1}} -> {"a.b": 1}; tuples become lists so values survive a JSON round trip."""
    out: dict[str, Any] = {}
    stack: list[tuple[str, Any]] = [(prefix, config)]
    while stack:
        path, node = stack.pop()
        for key, value in node.items():
            dotted = f"{path}{key}"
            if isinstance(value, dict):
                stack.append((dotted + ".", value))
            else:
                out[dotted] = list(value) if isinstance(value, tuple) else value
    return out


def diff_resolved(old: dict[str, Any], new: dict[str, Any]) -> dict[str, tuple[Any, Any]]:
    """Dotted paths whose values differ between two resolved configs -> (old value, new value)."""
    a, b = flatten_resolved(old), flatten_resolved(new)
    changed: dict[str, tuple[Any, Any]] = {}
    for key in sorted(a.keys() | b.keys()):
        if a.get(key) != b.get(key):
            changed[key] = (a.get(key), b.get(key))
    return changed
