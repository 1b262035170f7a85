"""Apply `[lora]` to a model (reference `src/engine/lora.py:52-171`).

Promotes the Linears of the configured `lora_target_groups()`, then leaves trainable only the
adapters, the model's `lora_required_trainable()` names, and (per switch) norms/LayerScale, the
input stem and the learned tokens. Returns a report of what was adapted, kept and frozen.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field

import torch.nn as nn

from ..layers.common.layer_scale import LayerScale
from ..layers.common.lora import adapted_modules, promote
from ..layers.common.rms_norm import RMSNorm
from ..models.base import BaseModel
from .config import LoRAConfig
from .optimizer import is_stem

logger = logging.getLogger(__name__)
NORM_TYPES = (nn.LayerNorm, nn.GroupNorm, RMSNorm, LayerScale)


@dataclass
class LoRAReport:
    adapted: list[str] = field(default_factory=list)
    trainable: list[str] = field(default_factory=list)
    frozen: list[str] = field(default_factory=list)
    adapter_params: int = 0
    trainable_params: int = 0
    total_params: int = 0

    def summary(self) -> str:
        frac = 100.0 * self.trainable_params / max(1, self.total_params)
        return (
            f"{len(self.adapted)} adapters, {self.adapter_params / 1e6:.2f}M adapter params; "
            f"{len(self.trainable)} of {len(self.trainable) + len(self.frozen)} tensors trainable "
            f"({self.trainable_params / 1e6:.2f}M of {self.total_params / 1e6:.1f}M params, {frac:.2f}%)"
        )


def _targets(model: BaseModel, config: LoRAConfig) -> list[nn.Linear]:
    groups = model.lora_target_groups()
    if not groups:
        raise ValueError(
            f"[lora] is enabled, but {type(model).__name__} declares no lora_target_groups(); there "
            "is nothing to adapt"
        )
    unknown = sorted(set(config.targets) - set(groups))
    if unknown:
        raise ValueError(
            f"[lora].targets names {unknown}, which {type(model).__name__} does not offer; its groups "
            f"are {sorted(groups)}"
        )
    out: list[nn.Linear] = []
    seen: set[int] = set()
    for name in config.targets:
        if not groups[name]:
            raise ValueError(f"[lora].targets names {name!r}, which is empty on this configuration")
        for m in groups[name]:
            if id(m) not in seen:
                seen.add(id(m))
                out.append(m)
    return out


def _keep(model: BaseModel, config: LoRAConfig) -> set[str]:
    names = dict(model.named_parameters())
    keep = {n for n in names if n.endswith((".lora_a", ".lora_b"))}
    required = model.lora_required_trainable()
    missing = sorted(n for n in required if n not in names)
    if missing:
        raise ValueError(
            f"{type(model).__name__}.lora_required_trainable() names {missing}, which is not a parameter"
        )
    keep |= set(required)
    if config.train_norms:
        for prefix, module in model.named_modules():
            if isinstance(module, NORM_TYPES):
                keep |= {f"{prefix}.{n}" if prefix else n for n, _ in module.named_parameters(recurse=False)}
    for n in names:
        if config.train_stem and is_stem(n):
            keep.add(n)
        if config.train_tokens and (n.endswith("_token") or "tokens" in n):
            keep.add(n)
    return keep


def apply_lora(model: BaseModel, config: LoRAConfig) -> LoRAReport:
    for module in _targets(model, config):
        promote(module, rank=config.rank, alpha=config.alpha)
    keep = _keep(model, config)
    report = LoRAReport(adapted=[n for n, _ in adapted_modules(model)])
    for name, p in model.named_parameters():
        trainable = name in keep
        p.requires_grad_(trainable)
        report.total_params += p.numel()
        if trainable:
            report.trainable.append(name)
            report.trainable_params += p.numel()
        else:
            report.frozen.append(name)
        if name.endswith((".lora_a", ".lora_b")):
            report.adapter_params += p.numel()
    if not report.trainable:
        raise ValueError("[lora] left no parameter trainable")
    logger.info("lora: %s", report.summary())
    return report
