"""AdamW over (lr multiplier, wd multiplier) parameter groups, and the warmup/decay schedule.

The `[trainer]` keys and their meaning are the reference's (`src/engine/optimizer.py:17-251`); the
code is this framework's own. Every trainable parameter gets a role from its dotted name:

* `stem`  -- the input adapter (`patch_embed`, `pos_embed`, `patch_proj`, `level_embed`) and learned
  tokens (`*_token`, `*tokens*`): depth 0;
* `block` -- inside `blocks.<i>.`: depth i + 1;
* `top`   -- everything above the stack (final norms, heads) and, when the root is an algorithm,
  every parameter outside its backbone (`model.`): depth n_blocks + 1, never discounted.

The learning-rate multiplier is `layerwise_lr_decay ** (n_blocks + 1 - depth)` (times
`patch_embed_lr_mult` on the patch projection); weight decay is off for LoRA factors and for
parameters of rank < 2 when those switches are on. Parameters with equal multipliers share one
AdamW group. The schedule is a linear warmup, then linear or cosine decay to `min_lr_ratio`, times
the unfreeze ramp; weight decay follows its own cosine from `weight_decay` to `final_weight_decay`.

`build_optimizer` returns `torch.optim.AdamW` unless the fused optimizer is requested and
available; `FusedAdamW` (in `fused_adamw.py`) keeps AdamW's update rule and its
`exp_avg`/`exp_avg_sq`/`step` state layout, so checkpoints interchange.
"""

from __future__ import annotations

import math
import re
from collections import defaultdict
from typing import Any

import torch
import torch.nn as nn
from torch.optim import AdamW, Optimizer
from torch.optim.lr_scheduler import LambdaLR

from .config import LR_SCHEDULES, TrainerConfig

_BLOCK = re.compile(r"(?:^|\.)blocks\.(\d+)\.")
STEM_NAMES = ("patch_embed", "pos_embed", "patch_proj", "level_embed")
_PATCH_PROJECTIONS = ("patch_embed", "patch_proj")
_BACKBONE = "model."


def is_stem(name: str) -> bool:
    """True for the input adapter's parameters (also what the frozen-backbone warm-up keeps trainable)."""
    return any(part in name for part in STEM_NAMES)


def _block_of(name: str) -> int | None:
    hit = _BLOCK.search(name)
    return None if hit is None else int(hit.group(1))


def parameter_depth(name: str, n_blocks: int, backbone_scoped: bool = False) -> int:
    """0 for the stem and tokens, i + 1 inside block i, n_blocks + 1 above the stack."""
    top = n_blocks + 1
    if backbone_scoped and not name.startswith(_BACKBONE):
        return top
    block = _block_of(name)
    if block is not None:
        return block + 1
    learned_token = name.endswith("_token") or "tokens" in name
    return 0 if (is_stem(name) or learned_token) else top


def lr_scale(name: str, n_blocks: int, config: TrainerConfig, backbone_scoped: bool = False) -> float:
    decay, patch_mult = config.layerwise_lr_decay, config.patch_embed_lr_mult
    if decay >= 1.0 and patch_mult == 1.0:
        return 1.0
    steps_below_top = n_blocks + 1 - parameter_depth(name, n_blocks, backbone_scoped)
    mult = decay**steps_below_top
    return mult * patch_mult if any(p in name for p in _PATCH_PROJECTIONS) else mult


def wd_scale(name: str, parameter: nn.Parameter, config: TrainerConfig) -> float:
    if config.zero_weight_decay_on_lora and (name.endswith(".lora_a") or name.endswith(".lora_b")):
        return 0.0
    if config.zero_weight_decay_on_norm_and_bias and parameter.dim() < 2:
        return 0.0
    return 1.0


def build_param_groups(model: nn.Module, config: TrainerConfig) -> list[dict[str, Any]]:
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    if not named:
        raise ValueError("nothing to optimise: no parameter of the model requires a gradient")
    blocks = [b for n, _ in model.named_parameters() if (b := _block_of(n)) is not None]
    n_blocks = max(blocks) + 1 if blocks else 0
    scoped = any(n.startswith(_BACKBONE) for n, _ in model.named_parameters())
    members: dict[tuple[float, float], list[nn.Parameter]] = defaultdict(list)
    for name, param in named:
        members[(lr_scale(name, n_blocks, config, scoped), wd_scale(name, param, config))].append(param)
    groups = []
    for lr_mult, wd_mult in sorted(members, reverse=True):
        groups.append({
            "params": members[(lr_mult, wd_mult)],
            "lr": config.lr * lr_mult,
            "weight_decay": config.weight_decay * wd_mult,
            "lr_multiplier": lr_mult,
            "wd_multiplier": wd_mult,
        })
    return groups


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
    """Fraction of the decayable range left after `progress` (0..1) of the decay phase."""
    shapes = {"cosine": lambda t: (1.0 + math.cos(math.pi * t)) / 2.0, "linear": lambda t: 1.0 - t}
    if schedule not in shapes:
        raise ValueError(f"lr_schedule {schedule!r} is not one of {list(LR_SCHEDULES)}")
    return shapes[schedule](progress)


def unfreeze_ramp(step: int, config: TrainerConfig) -> float:
    """Linear ramp of the learning rate over `unfreeze_warmup_steps` after the backbone unfreezes."""
    ramp = config.unfreeze_warmup_steps
    since = step - config.freeze_backbone_steps
    if config.freeze_backbone_steps > 0 and ramp > 0 and 0 <= since < ramp:
        return (since + 1) / ramp
    return 1.0


def lr_multiplier(step: int, config: TrainerConfig) -> float:
    """Learning rate at `step` as a fraction of the configured peak."""
    warm = config.warmup_steps
    if warm > 0 and step < warm:
        return (step + 1) / warm
    t = (step - warm) / max(1, config.max_steps - warm)
    floor = config.min_lr_ratio
    shaped = floor + (1.0 - floor) * decay_fraction(min(max(t, 0.0), 1.0), config.lr_schedule)
    return shaped * unfreeze_ramp(step, config)


def weight_decay_at(step: int, config: TrainerConfig) -> float:
    """Weight decay at `step`: constant, or a cosine from `weight_decay` to `final_weight_decay`."""
    start, end = config.weight_decay, config.final_weight_decay
    if end is None:
        return start
    t = min(max(step / max(1, config.max_steps), 0.0), 1.0)
    return end + (start - end) * decay_fraction(t, "cosine")


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
