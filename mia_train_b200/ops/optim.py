"""Multi-tensor optimizer kernels: global grad norm, in-place scaling, and the fused AdamW update.

Each op is one launch over a device table of tensor pointers (built once per parameter set and
cached, so that a captured CUDA graph replays it). Nothing here synchronises with the host: the
clip coefficient `min(1, max_norm / (norm + 1e-6))` is computed on the device and handed to the
AdamW kernel, which scales gradients as it reads them instead of rewriting them first.
"""

from __future__ import annotations

import torch

from ._native import native


def grad_sumsq(tensors: list[torch.Tensor]) -> torch.Tensor:
    out = torch.zeros((), device=tensors[0].device, dtype=torch.float32)
    native().multi_tensor_sumsq(tensors, out)
    return out


def clip_coefficient(total_norm: torch.Tensor, max_norm: float) -> torch.Tensor:
    return torch.clamp(max_norm / (total_norm + 1e-6), max=1.0)


def clip_grad_norm_native(params: list[torch.nn.Parameter], max_norm: float) -> torch.Tensor:
    grads = [p.grad for p in params]
    norm = grad_sumsq(grads).sqrt()
    coef = clip_coefficient(norm, max_norm)
    native().multi_tensor_scale(grads, coef)
    return norm


def adamw_step(
    params: list[torch.Tensor],
    grads: list[torch.Tensor],
    exp_avgs: list[torch.Tensor],
    exp_avg_sqs: list[torch.Tensor],
    steps: list[torch.Tensor],
    group_index: torch.Tensor,
    hyper: torch.Tensor,
    eps: float,
    grad_scale: torch.Tensor | None,
    shadows: list[torch.Tensor] | None = None,
) -> None:
    """One AdamW update for every tensor; `hyper[g] = (lr, weight_decay, beta1, beta2)` per group.

    Steps are incremented in the kernel; bias corrections use the incremented step, as
    `torch.optim.AdamW` does. `shadows[i]` (an empty tensor for none) receives the updated
    parameter in bf16.
    """
    native().adamw_step(
        params, grads, exp_avgs, exp_avg_sqs, steps, group_index, hyper, float(eps), grad_scale, shadows or []
    )


def adamw_reference(
    param: torch.Tensor,
    grad: torch.Tensor,
    exp_avg: torch.Tensor,
    exp_avg_sq: torch.Tensor,
    step: int,
    lr: float,
    weight_decay: float,
    beta1: float,
    beta2: float,
    eps: float,
) -> None:
    """torch.optim.AdamW's update for one tensor, written out (the oracle for the kernel tests)."""
    param.mul_(1 - lr * weight_decay)
    exp_avg.lerp_(grad, 1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)
    bc1 = 1 - beta1**step
    bc2 = 1 - beta2**step
    denom = (exp_avg_sq.sqrt() / (bc2**0.5)).add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)


@torch.no_grad()
def ema_update(teacher: list[torch.Tensor], student: list[torch.Tensor], momentum: float) -> None:
    """teacher <- momentum * teacher + (1 - momentum) * student, one launch for all tensors on CUDA."""
    if not teacher:
        return
    from ._native import use_native

    plain = all(type(t) is torch.Tensor and t.dtype == torch.float32 and t.is_contiguous() for t in teacher + student)
    if plain and use_native(teacher[0]):
        native().ema_update(teacher, student, float(momentum))
        return
    torch._foreach_mul_(teacher, momentum)
    torch._foreach_add_(teacher, student, alpha=1 - momentum)
