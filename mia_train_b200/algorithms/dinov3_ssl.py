"""`dinov3`: the DINOv3 self-supervised objective (reference `src/algorithms/dinov3_ssl.py:51-360`).

Student (`student.backbone`, `student.dino_head`, `student.ibot_head`) and an EMA teacher (a
frozen copy). Per step: 2 global + `n_local_crops` local views made on the device; iBOT block
masks on the global grid; the teacher's class-token and masked-patch logits are centred with
Sinkhorn-Knopp; the student sees masked global views and unmasked local views; the loss is the
DINO term (global pairs without the diagonal, weighted with the local pairs by their counts), the
iBOT term and KoLeo on the pre-head class tokens. The teacher temperature warms up linearly and
the teacher momentum follows a cosine from `momentum_teacher` to `final_momentum_teacher` over
`total_steps`; both read a `_step` buffer that is checkpointed with the model.

The reference defines `update_teacher` but its engine never calls it, so its teacher stays the
initial student. Here the engine calls `after_optimizer_step`, which applies the EMA with one
native multi-tensor kernel (teacher params are fp32 tensors matched one-to-one with the
student's); under FSDP the shards are updated in place.
"""

from __future__ import annotations

import copy
import math
from typing import Any

import torch
import torch.nn as nn

from ..data.base import BaseDataset
from ..layers.dinov3.head import DINOHead
from ..ops.optim import ema_update
from .base import BaseAlgorithm
from .dinov3.losses import DINOLoss, IBOTPatchLoss, KoLeoLoss
from .dinov3.multicrop import AugmentationConfig, block_mask, photometric, random_resized_crop
from .registry import AlgorithmRegistry


def _local(t: torch.Tensor) -> torch.Tensor:
    to_local = getattr(t, "to_local", None)
    return to_local() if to_local is not None else t


@AlgorithmRegistry.register("dinov3")
class DINOv3(BaseAlgorithm):
    _step: torch.Tensor

    def __init__(
        self,
        model: nn.Module,
        dataset: BaseDataset | None = None,
        total_steps: int = 100_000,
        input_axes: str | None = None,
        input_key: str = "img",
        global_crop_size: int = 64,
        local_crop_size: int = 32,
        n_local_crops: int = 8,
        global_crop_scale: tuple[float, float] = (0.32, 1.0),
        local_crop_scale: tuple[float, float] = (0.05, 0.32),
        head_n_prototypes: int = 65536,
        head_bottleneck_dim: int = 256,
        head_hidden_dim: int = 2048,
        head_nlayers: int = 3,
        student_temp: float = 0.1,
        teacher_temp: float = 0.07,
        warmup_teacher_temp: float = 0.04,
        warmup_teacher_temp_steps: int = 30_000,
        momentum_teacher: float = 0.992,
        final_momentum_teacher: float = 1.0,
        dino_loss_weight: float = 1.0,
        ibot_loss_weight: float = 1.0,
        koleo_loss_weight: float = 0.1,
        global_ignore_diagonal: bool = True,
        mask_ratio_min_max: tuple[float, float] = (0.1, 0.5),
        mask_sample_probability: float = 0.5,
        augmentation: dict[str, Any] | None = None,
        update_teacher_every_step: bool = True,
    ) -> None:
        super().__init__(model, dataset)
        for name, value in (("head_n_prototypes", head_n_prototypes), ("total_steps", total_steps)):
            if value < 1:
                raise ValueError(f"{name} must be >= 1, got {value}")
        if not hasattr(model, "forward_features"):
            raise TypeError(
                f"{type(model).__name__} has no forward_features, so it cannot be trained with DINOv3; use a "
                "dinov3_vit or dinov3_vit3d encoder"
            )
        self.input_axes = self.resolve_input_axes(input_axes, dataset)
        self.input_key = input_key
        self.total_steps = total_steps
        self.n_local_crops = n_local_crops
        self.global_crop_scale = tuple(global_crop_scale)
        self.local_crop_scale = tuple(local_crop_scale)
        self.mask_ratio_min_max = tuple(mask_ratio_min_max)
        self.mask_sample_probability = mask_sample_probability
        self.augmentation = AugmentationConfig(**(augmentation or {}))
        self.teacher_temp = teacher_temp
        self.warmup_teacher_temp = warmup_teacher_temp
        self.warmup_teacher_temp_steps = warmup_teacher_temp_steps
        self.momentum_teacher = momentum_teacher
        self.final_momentum_teacher = final_momentum_teacher
        self.dino_loss_weight = dino_loss_weight
        self.ibot_loss_weight = ibot_loss_weight
        self.koleo_loss_weight = koleo_loss_weight
        self.global_ignore_diagonal = global_ignore_diagonal
        self.update_teacher_every_step = update_teacher_every_step
        rank = int(getattr(model, "spatial_rank", 3))
        self.spatial_rank = rank
        self.global_crop_size = (global_crop_size,) * rank
        self.local_crop_size = (local_crop_size,) * rank
        patch = model.patch_size if isinstance(model.patch_size, int) else int(model.patch_size[0])
        self.global_grid = tuple(s // patch for s in self.global_crop_size)
        embed_dim = int(model.embed_dim)

        def head() -> DINOHead:
            h = DINOHead(embed_dim, head_n_prototypes, nlayers=head_nlayers, hidden_dim=head_hidden_dim,
                         bottleneck_dim=head_bottleneck_dim)
            h.init_weights()
            return h

        self.student = nn.ModuleDict({"backbone": model, "dino_head": head(), "ibot_head": head()})
        self.teacher = copy.deepcopy(self.student)
        for p in self.teacher.parameters():
            p.requires_grad_(False)
        self.dino_loss = DINOLoss(head_n_prototypes, student_temp=student_temp)
        self.ibot_loss = IBOTPatchLoss(head_n_prototypes, student_temp=student_temp)
        self.koleo_loss = KoLeoLoss()
        self.register_buffer("_step", torch.zeros((), dtype=torch.long))
        # host copy of `_step` (value, buffer identity, in-place version), so the schedules never read
        # the device; any other write to the buffer (a checkpoint load, a measurement step that
        # restores buffers) changes its identity or version and forces one read
        self._host_step: tuple[int, int, int] | None = None

    # -- schedules ----------------------------------------------------------------------------
    @property
    def step(self) -> int:
        buf = self._step
        cached = self._host_step
        if cached is None or cached[1] != id(buf) or cached[2] != buf._version:
            cached = (int(buf.item()), id(buf), buf._version)
            self._host_step = cached
        return cached[0]

    def current_teacher_temp(self, step: int | None = None) -> float:
        step = self.step if step is None else step
        if self.warmup_teacher_temp_steps <= 0:
            return self.teacher_temp
        progress = min(1.0, step / self.warmup_teacher_temp_steps)
        return self.warmup_teacher_temp + progress * (self.teacher_temp - self.warmup_teacher_temp)

    def current_momentum(self, step: int | None = None) -> float:
        step = self.step if step is None else step
        progress = min(1.0, step / max(1, self.total_steps))
        span = self.final_momentum_teacher - self.momentum_teacher
        return self.final_momentum_teacher - span * (1 + math.cos(math.pi * progress)) / 2

    @torch.no_grad()
    def update_teacher(self, momentum: float | None = None) -> None:
        m = self.current_momentum() if momentum is None else momentum
        teacher = [_local(p.data) for p in self.teacher.parameters()]
        student = [_local(p.data) for p in self.student.parameters()]
        ema_update(teacher, student, m)

    def after_optimizer_step(self, step: int) -> None:
        if self.update_teacher_every_step:
            self.update_teacher()

    def train(self, mode: bool = True) -> DINOv3:
        super().train(mode)
        self.teacher.eval()
        return self

    def checkpointable_modules(self) -> tuple[nn.Module, ...]:
        return ()

    def extra_tensor_parallel_models(self) -> tuple[nn.Module, ...]:
        """The teacher backbone takes the student's tensor-parallel layout, so the EMA pairs
        matching shards."""
        return (self.teacher["backbone"],)

    def extra_sharded_modules(self) -> tuple[nn.Module, ...]:
        """Shard the teacher backbone and heads as their own FSDP units (used by parallelize)."""
        return (self.teacher,)

    # -- step -----------------------------------------------------------------------------------
    def _make_views(self, volumes: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        a = self.augmentation

        def view(size, scale):
            crop = random_resized_crop(volumes, size, scale, flip_prob=a.flip_prob, rotate_prob=a.rotate_prob)
            return photometric(crop, a)

        globals_ = [view(self.global_crop_size, self.global_crop_scale) for _ in range(2)]
        locals_ = [view(self.local_crop_size, self.local_crop_scale) for _ in range(self.n_local_crops)]
        return torch.cat(globals_, dim=0), torch.cat(locals_, dim=0)

    @staticmethod
    def _colsum_buffer(head: nn.Module, x: torch.Tensor) -> torch.Tensor:
        return torch.zeros(head.last_layer.weight.shape[0], device=x.device, dtype=torch.float32)

    def _step_impl(self, batch: Any, train: bool) -> dict[str, torch.Tensor]:
        backbone = self.student["backbone"]
        volumes = backbone.prepare_input(batch[self.input_key], self.input_axes)
        global_views, local_views = self._make_views(volumes)
        b = volumes.shape[0]
        # the masks are drawn on the host: their count and the masked token indices are known there,
        # so the step selects masked tokens with index_select and never waits on the device
        masks_host = block_mask(self.global_grid, 2 * b, self.mask_ratio_min_max,
                                sample_probability=self.mask_sample_probability)
        n_masked = int(masks_host.sum())
        masked_idx_host = masks_host.flatten().nonzero().squeeze(1)
        if volumes.is_cuda:
            masks = masks_host.pin_memory().to(volumes.device, non_blocking=True)
            masked_idx = masked_idx_host.pin_memory().to(volumes.device, non_blocking=True)
        else:
            masks, masked_idx = masks_host.to(volumes.device), masked_idx_host.to(volumes.device)
        temp = self.current_teacher_temp()
        with torch.no_grad():
            t_out = self.teacher["backbone"].forward_features(global_views)
            # on CUDA the prototype GEMMs also produce Sinkhorn's first column sums in their epilogue
            fused = t_out["x_norm_clstoken"].is_cuda
            cls_sum = self._colsum_buffer(self.teacher["dino_head"], t_out["x_norm_clstoken"]) if fused else None
            t_cls_logits = self.teacher["dino_head"](t_out["x_norm_clstoken"], cls_sum, temp) if fused else \
                self.teacher["dino_head"](t_out["x_norm_clstoken"])
            t_cls_probs = self.dino_loss.sinkhorn_knopp_teacher(t_cls_logits, temp, colsum=cls_sum).unflatten(0, (2, b))
            if n_masked > 0:
                masked_teacher = t_out["x_norm_patchtokens"].flatten(0, 1).index_select(0, masked_idx)
                patch_sum = self._colsum_buffer(self.teacher["ibot_head"], masked_teacher) if fused else None
                patch_logits = self.teacher["ibot_head"](masked_teacher, patch_sum, temp) if fused else \
                    self.teacher["ibot_head"](masked_teacher)
                t_patch_probs = self.ibot_loss.sinkhorn_knopp_teacher(
                    patch_logits, temp, n_masked_patches=n_masked, colsum=patch_sum
                )
        s_global, s_local = backbone.forward_features([global_views, local_views], [masks, None])
        head = self.student["dino_head"]
        s_global_cls = head(s_global["x_norm_clstoken"])
        s_local_cls = head(s_local["x_norm_clstoken"])
        g_terms = 2 if self.global_ignore_diagonal else 4
        l_terms = 2 * self.n_local_crops
        total = g_terms + l_terms
        dino_global = self.dino_loss(s_global_cls.unflatten(0, (2, b)), t_cls_probs,
                                     ignore_diagonal=self.global_ignore_diagonal)
        dino_local = self.dino_loss(s_local_cls.unflatten(0, (self.n_local_crops, b)), t_cls_probs)
        loss = self.dino_loss_weight * (dino_global * (g_terms / total) + dino_local * (l_terms / total))
        metrics = {"dino_global": dino_global.detach(), "dino_local": dino_local.detach()}
        if n_masked > 0:
            s_masked = self.student["ibot_head"](s_global["x_norm_patchtokens"].flatten(0, 1).index_select(0, masked_idx))
            ibot = self.ibot_loss.forward_masked(s_masked, t_patch_probs, masks, n_masked_patches=n_masked)
            loss = loss + self.ibot_loss_weight * ibot
            metrics["ibot"] = ibot.detach()
        if self.koleo_loss_weight > 0:
            pre = s_global["x_norm_clstoken"].unflatten(0, (2, b))
            koleo = (self.koleo_loss(pre[0]) + self.koleo_loss(pre[1])) / 2
            loss = loss + self.koleo_loss_weight * 2 * koleo
            metrics["koleo"] = koleo.detach()
        if train:
            host_step = self.step
            self._step += 1
            self._host_step = (host_step + 1, id(self._step), self._step._version)
        momentum = self.current_momentum()
        metrics["loss"] = loss
        metrics["teacher_temp"] = torch.full((), temp, device=loss.device)
        metrics["teacher_momentum"] = torch.full((), momentum, device=loss.device)
        metrics["masked_fraction"] = torch.full((), n_masked / masks_host.numel(), device=loss.device)
        return metrics

    def training_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step_impl(batch, train=True)

    def validation_step(self, batch: Any) -> dict[str, torch.Tensor]:
        return self._step_impl(batch, train=False)
