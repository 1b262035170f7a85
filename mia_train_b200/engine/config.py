"""Strict dataclasses for the `[init]`, `[lora]`, `[augment]` and `[trainer]` TOML sections.

Field names, defaults and validation follow the reference's `src/engine/config.py:17-417`, so a
config written for the reference loads here unchanged. New `[trainer]` keys: `fused_optimizer` (this
framework's CUDA AdamW over fp32 master weights), `nan_guard` (stop on a non-finite loss),
`watchdog_seconds` (dump stacks when a step hangs), `step_mode` (`"graph"` replays the whole step
from one CUDA graph) and `graph_dp` (the data-parallel gradient path of the graph step).
"""

from __future__ import annotations

from dataclasses import dataclass

from ..data.augment import ROTATIONS

PRECISIONS = ("fp32", "bf16")
LR_SCHEDULES = ("linear", "cosine")


@dataclass(frozen=True)
class InitConfig:
    """Where the model's weights start when not from scratch (reference `engine/config.py:17-84`).

    `target="model"` loads the bare encoder before the algorithm wraps it; `"algorithm"` loads the
    whole strategy (decoder/head included). `merge_lora` folds adapters in the checkpoint into their
    base weights before matching.
    """

    path: str = ""
    prefix: str = ""
    inflate_2d_to_3d: bool = False
    skip: tuple[str, ...] = ()
    strict: bool = True
    allow_unused: bool = False
    target: str = "model"
    merge_lora: bool = False

    def __post_init__(self) -> None:
        if self.target not in ("model", "algorithm"):
            raise ValueError(f"[init].target must be 'model' or 'algorithm', got {self.target!r}")
        if not self.path and (
            self.prefix
            or self.inflate_2d_to_3d
            or self.skip
            or self.allow_unused
            or self.merge_lora
            or self.target != "model"
        ):
            raise ValueError(
                "[init] sets loading options but no 'path', so nothing would be loaded and the run "
                "would silently start from scratch"
            )
        object.__setattr__(self, "skip", tuple(self.skip))


@dataclass(frozen=True)
class LoRAConfig:
    """Low-rank adaptation of a pretrained encoder (reference `engine/config.py:87-159`).

    `rank=0` disables it. The delta is scaled by `alpha/rank`, so `alpha` has no default.
    """

    rank: int = 0
    alpha: float = 0.0
    targets: tuple[str, ...] = ("attn_qkv", "attn_proj")
    train_stem: bool = True
    train_norms: bool = True
    train_tokens: bool = True

    def enabled(self) -> bool:
        return self.rank > 0

    def __post_init__(self) -> None:
        object.__setattr__(self, "targets", tuple(self.targets))
        if self.rank < 0:
            raise ValueError(f"[lora].rank must be >= 0, got {self.rank}; 0 disables")
        if not self.enabled():
            if self.alpha or not self.targets:
                raise ValueError(
                    "[lora] sets options but leaves rank at 0, so no adapter would be built; set "
                    "rank, or drop the section"
                )
            return
        if self.alpha <= 0.0:
            raise ValueError(
                f"[lora].alpha must be > 0 when rank is set, got {self.alpha}; with rank = "
                f"{self.rank}, alpha = {2 * self.rank} gives the common scaling of 2"
            )
        if not self.targets:
            raise ValueError("[lora].targets is empty; name at least one lora_target_groups() entry")
        repeated = sorted({t for t in self.targets if self.targets.count(t) > 1})
        if repeated:
            raise ValueError(f"[lora].targets repeats {repeated}")


@dataclass(frozen=True)
class AugmentConfig:
    """Training-only volumetric augmentation (reference `engine/config.py:162-210`). Off by default."""

    rotate: str = "none"
    drop_slice_prob: float = 0.0
    shift_slice_prob: float = 0.0
    shift_magnitude: int = 10
    intensity: bool = False
    mul_intensity: float = 0.1
    add_intensity: float = 0.1
    noise_scale: float = 0.0

    def __post_init__(self) -> None:
        if self.rotate not in ROTATIONS:
            raise ValueError(f"[augment].rotate must be one of {ROTATIONS}, got {self.rotate!r}")

    def enabled(self) -> bool:
        return bool(
            self.rotate != "none"
            or self.drop_slice_prob > 0.0
            or (self.shift_slice_prob > 0.0 and self.shift_magnitude > 0)
            or self.intensity
            or self.noise_scale > 0.0
        )


@dataclass(frozen=True)
class TrainerConfig:
    """Training-loop hyperparameters (reference `engine/config.py:213-417`)."""

    max_steps: int
    batch_size: int
    lr: float = 1e-3
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    warmup_steps: int = 0
    min_lr_ratio: float = 0.0
    grad_clip_norm: float | None = 1.0
    lr_schedule: str = "linear"
    layerwise_lr_decay: float = 1.0
    patch_embed_lr_mult: float = 1.0
    final_weight_decay: float | None = None
    zero_weight_decay_on_norm_and_bias: bool = True
    zero_weight_decay_on_lora: bool = True
    activation_checkpointing: bool = False
    peak_tflops: float | None = None
    measure_mfu: bool = True
    profile: bool = False
    profile_start_step: int = 50
    profile_steps: int = 6
    profile_all_ranks: bool = False
    profile_memory: bool = False
    freeze_backbone_steps: int = 0
    unfreeze_warmup_steps: int = 1000
    precision: str = "fp32"
    log_every: int = 10
    checkpoint_every: int = 0
    val_every: int = 0
    num_workers: int = 0
    persistent_workers: bool = False
    prefetch_factor: int = 2
    seed: int = 0
    # New in this framework. The fused AdamW is this framework's multi-tensor CUDA kernel over
    # fp32 master weights; "auto" uses it whenever the native extension is loaded on a CUDA device.
    fused_optimizer: str = "auto"
    # Abort the run when the loss goes non-finite, after saving nothing (the reference has no guard).
    nan_guard: bool = True
    # Seconds a step may take before the watchdog thread dumps every thread's stack (0 = off).
    watchdog_seconds: float = 0.0
    # "eager" runs the reference loop; "graph" captures forward, backward, clip, AdamW and the
    # schedule into one CUDA graph (engine/graph_step.py). The algorithm's step must then be free
    # of host synchronisation and shape changes (mae, simmim; not dinov3's variable mask counts).
    step_mode: str = "eager"
    # Data parallelism of the graph step across the dp ranks: "p2p" (sharded optimizer over peer
    # memory), "nccl" (the same over NCCL collectives) or "allreduce" (replicated optimizer).
    graph_dp: str = "p2p"

    def __post_init__(self) -> None:
        checks = [
            (self.max_steps >= 1, f"max_steps must be >= 1, got {self.max_steps}"),
            (self.batch_size >= 1, f"batch_size must be >= 1, got {self.batch_size}"),
            (self.lr > 0.0, f"lr must be > 0, got {self.lr}"),
            (self.warmup_steps >= 0, f"warmup_steps must be >= 0, got {self.warmup_steps}"),
            (
                self.warmup_steps < self.max_steps,
                f"warmup_steps ({self.warmup_steps}) must be < max_steps ({self.max_steps})",
            ),
            (0.0 <= self.min_lr_ratio <= 1.0, f"min_lr_ratio must be in [0, 1], got {self.min_lr_ratio}"),
            (
                self.grad_clip_norm is None or self.grad_clip_norm > 0.0,
                f"grad_clip_norm must be > 0 or None, got {self.grad_clip_norm}",
            ),
            (self.precision in PRECISIONS, f"precision must be one of {PRECISIONS}, got {self.precision!r}"),
            (
                self.lr_schedule in LR_SCHEDULES,
                f"lr_schedule must be one of {LR_SCHEDULES}, got {self.lr_schedule!r}",
            ),
            (self.log_every >= 1, f"log_every must be >= 1, got {self.log_every}"),
            (
                self.peak_tflops is None or self.peak_tflops > 0.0,
                f"peak_tflops must be > 0 or None, got {self.peak_tflops}",
            ),
            (self.num_workers >= 0, f"num_workers must be >= 0, got {self.num_workers}"),
            (self.prefetch_factor >= 1, f"prefetch_factor must be >= 1, got {self.prefetch_factor}"),
            (
                self.profile_start_step >= 0,
                f"profile_start_step must be >= 0, got {self.profile_start_step}",
            ),
            (
                self.profile_steps >= 1,
                f"profile_steps must be >= 1, got {self.profile_steps}; set profile = false instead",
            ),
            (
                self.freeze_backbone_steps >= 0,
                f"freeze_backbone_steps must be >= 0, got {self.freeze_backbone_steps}; 0 disables",
            ),
            (
                self.freeze_backbone_steps < self.max_steps,
                f"freeze_backbone_steps ({self.freeze_backbone_steps}) must be < max_steps "
                f"({self.max_steps}), or the backbone would never train",
            ),
            (
                self.unfreeze_warmup_steps >= 0,
                f"unfreeze_warmup_steps must be >= 0, got {self.unfreeze_warmup_steps}",
            ),
            (
                0.0 < self.layerwise_lr_decay <= 1.0,
                f"layerwise_lr_decay must be in (0, 1], got {self.layerwise_lr_decay}",
            ),
            (
                self.patch_embed_lr_mult > 0.0,
                f"patch_embed_lr_mult must be > 0, got {self.patch_embed_lr_mult}",
            ),
            (
                self.final_weight_decay is None or self.final_weight_decay >= 0.0,
                f"final_weight_decay must be >= 0 or None, got {self.final_weight_decay}",
            ),
            (
                self.fused_optimizer in ("auto", "on", "off"),
                f"fused_optimizer must be 'auto', 'on' or 'off', got {self.fused_optimizer!r}",
            ),
            (self.watchdog_seconds >= 0.0, f"watchdog_seconds must be >= 0, got {self.watchdog_seconds}"),
            (self.step_mode in ("eager", "graph"), f"step_mode must be 'eager' or 'graph', got {self.step_mode!r}"),
            (
                self.graph_dp in ("p2p", "nccl", "allreduce"),
                f"graph_dp must be 'p2p', 'nccl' or 'allreduce', got {self.graph_dp!r}",
            ),
        ]
        for ok, message in checks:
            if not ok:
                raise ValueError(message)
