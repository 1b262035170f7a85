"""AdamW over (lr multiplier, wd multiplier) parameter groups, and the warmup/decay schedule.

Grouping and schedule follow the reference's `src/engine/optimizer.py:17-251`:

* layerwise LR decay by block depth (`blocks.N.` in the name); the stem (`patch_embed`,
  `pos_embed`, `patch_proj`, `level_embed`) and tokens sit at depth 0, everything above the
  stack (final norms, heads, an algorithm's decoder) is not discounted; only parameters under
  `model.` have a depth when the root is an algorithm;
* `patch_embed_lr_mult` on the patch projection;
* weight decay exempted by rank (ndim < 2) and for LoRA factors;
* linear warmup, then linear or cosine decay to `min_lr_ratio`, times an unfreeze ramp; weight decay
  follows its own cosine from `weight_decay` to `final_weight_decay`.

`build_optimizer` returns `torch.optim.AdamW` unless the fused optimizer is requested and
available; `FusedAdamW` (in `fused_adamw.py`) keeps AdamW's update rule and its
`exp_avg`/`exp_avg_sq`/`step` state layout, so checkpoints interchange.
"""

from __future__ import annotations

import math
import re
from typing import Any

import torch
import torch.nn as nn
from torch.optim import AdamW, Optimizer
from torch.optim.lr_scheduler import LambdaLR

from .config import LR_SCHEDULES, TrainerConfig

_BLOCK_INDEX = re.compile(r"(?:^|\.)blocks\.(\d+)\.")
_STEM_MARKERS = ("patch_embed", "pos_embed", "patch_proj", "level_embed")
_BACKBONE_PREFIX = "model."


def is_stem(name: str) -> bool:
    return any(marker in name for marker in _STEM_MARKERS)


def _block_count(model: nn.Module) -> int:
    depths = [int(m.group(1)) for name, _ in model.named_parameters() if (m := _BLOCK_INDEX.search(name))]
    return max(depths) + 1 if depths else 0


def parameter_depth(name: str, n_blocks: int, backbone_scoped: bool = False) -> int:
    if backbone_scoped and not name.startswith(_BACKBONE_PREFIX):
        return n_blocks + 1
    match = _BLOCK_INDEX.search(name)
    if match is not None:
        return int(match.group(1)) + 1
    if is_stem(name) or name.endswith("_token") or "tokens" in name:
        return 0
    return n_blocks + 1


def lr_scale(name: str, n_blocks: int, config: TrainerConfig, backbone_scoped: bool = False) -> float:
    if config.layerwise_lr_decay >= 1.0 and config.patch_embed_lr_mult == 1.0:
        return 1.0
    depth = parameter_depth(name, n_blocks, backbone_scoped)
    scale = config.layerwise_lr_decay ** (n_blocks + 1 - depth)
    if "patch_embed" in name or "patch_proj" in name:
        scale *= config.patch_embed_lr_mult
    return scale


def wd_scale(name: str, parameter: nn.Parameter, config: TrainerConfig) -> float:
    if name.endswith((".lora_a", ".lora_b")) and config.zero_weight_decay_on_lora:
        return 0.0
    if not config.zero_weight_decay_on_norm_and_bias:
        return 1.0
    return 0.0 if parameter.ndim < 2 else 1.0


def build_param_groups(model: nn.Module, config: TrainerConfig) -> list[dict[str, Any]]:
    n_blocks = _block_count(model)
    scoped = any(name.startswith(_BACKBONE_PREFIX) for name, _ in model.named_parameters())
    buckets: dict[tuple[float, float], dict[str, Any]] = {}
    for name, parameter in model.named_parameters():
        if not parameter.requires_grad:
            continue
        key = (lr_scale(name, n_blocks, config, scoped), wd_scale(name, parameter, config))
        group = buckets.setdefault(
            key,
            {
                "params": [],
                "lr": config.lr * key[0],
                "weight_decay": config.weight_decay * key[1],
                "lr_multiplier": key[0],
                "wd_multiplier": key[1],
            },
        )
        group["params"].append(parameter)
    if not buckets:
        raise ValueError("model has no parameters that require grad, so there is nothing to train")
    return [buckets[key] for key in sorted(buckets, reverse=True)]


def _fused_wanted(config: TrainerConfig, model: nn.Module) -> bool:
    if config.fused_optimizer == "off":
        return False
    params = [p for p in model.parameters() if p.requires_grad]
    on_cuda = bool(params) and all(p.is_cuda for p in params)
    try:
        from torch.distributed.tensor import DTensor

        sharded = any(isinstance(p, DTensor) for p in params)
    except ImportError:  # pragma: no cover
        sharded = False
    if config.fused_optimizer == "on":
        if not on_cuda:
            raise ValueError("[trainer].fused_optimizer = 'on' needs every parameter on a CUDA device")
        return True
    return on_cuda and not sharded


def build_optimizer(model: nn.Module, config: TrainerConfig) -> Optimizer:
    groups = build_param_groups(model, config)
    if _fused_wanted(config, model):
        from .fused_adamw import FusedAdamW

        return FusedAdamW(groups, lr=config.lr, betas=(config.beta1, config.beta2), weight_decay=config.weight_decay)
    return AdamW(groups, lr=config.lr, betas=(config.beta1, config.beta2), weight_decay=config.weight_decay)


def decay_fraction(progress: float, schedule: str) -> float:
    if schedule == "cosine":
        return 0.5 * (1.0 + math.cos(math.pi * progress))
    if schedule == "linear":
        return 1.0 - progress
    raise ValueError(f"unknown lr_schedule {schedule!r}; expected one of {list(LR_SCHEDULES)}")


def unfreeze_ramp(step: int, config: TrainerConfig) -> float:
    if config.freeze_backbone_steps <= 0 or config.unfreeze_warmup_steps <= 0:
        return 1.0
    offset = step - config.freeze_backbone_steps
    if offset < 0 or offset >= config.unfreeze_warmup_steps:
        return 1.0
    return (offset + 1) / config.unfreeze_warmup_steps


def lr_multiplier(step: int, config: TrainerConfig) -> float:
    if config.warmup_steps > 0 and step < config.warmup_steps:
        return (step + 1) / config.warmup_steps
    span = max(1, config.max_steps - config.warmup_steps)
    progress = min(1.0, max(0.0, (step - config.warmup_steps) / span))
    value = config.min_lr_ratio + (1.0 - config.min_lr_ratio) * decay_fraction(progress, config.lr_schedule)
    return value * unfreeze_ramp(step, config)


def weight_decay_at(step: int, config: TrainerConfig) -> float:
    if config.final_weight_decay is None:
        return config.weight_decay
    progress = min(1.0, max(0.0, step / max(1, config.max_steps)))
    span = config.final_weight_decay - config.weight_decay
    return config.weight_decay + span * (1.0 - math.cos(math.pi * progress)) / 2


class WarmupDecaySchedule(LambdaLR):
    """LambdaLR over `lr_multiplier`, also rewriting each group's weight decay every step."""

    def __init__(self, optimizer: Optimizer, config: TrainerConfig) -> None:
        self._config = config
        super().__init__(optimizer, lr_lambda=lambda step: lr_multiplier(step, config))
        self._apply_weight_decay()

    def _apply_weight_decay(self) -> None:
        decay = weight_decay_at(self.last_epoch, self._config)
        for group in self.optimizer.param_groups:
            group["weight_decay"] = decay * group.get("wd_multiplier", 1.0)

    def step(self, epoch: int | None = None) -> None:  # type: ignore[override]
        super().step(epoch)
        self._apply_weight_decay()


def build_lr_scheduler(optimizer: Optimizer, config: TrainerConfig) -> LambdaLR:
    return WarmupDecaySchedule(optimizer, config)


def clip_grad_norm_(parameters: Any, max_norm: float) -> torch.Tensor:
    """Global L2 clip; the native multi-tensor norm when every grad is a plain CUDA tensor."""
    params = [p for p in parameters if p.grad is not None]
    if params and all(p.grad.is_cuda and type(p.grad) is torch.Tensor for p in params):
        from ..ops.optim import clip_grad_norm_native

        return clip_grad_norm_native(params, max_norm)
    return torch.nn.utils.clip_grad_norm_(params, max_norm)
