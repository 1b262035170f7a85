"""Masked-autoencoding token plumbing and loss on native kernels.

* `restore_with_mask_token(visible, mask_token, restore)` -- the decoder input: `visible` (B, K, d)
  followed by `N - K` copies of the mask token, permuted back to grid order by `restore` (B, N).
  One gather kernel replaces the reference's expand + cat + gather (`src/algorithms/mae.py:116-132`);
  its backward scatters the visible rows back and sums the mask-token gradient.
* `norm_pix_mse(prediction, volumes, mask, patch)` -- per masked patch, normalise the target
  patch by its own mean and unbiased variance (+1e-6), take the squared error against the
  prediction, average over the patch and then over masked patches (reference
  `src/algorithms/mae.py:155-163`). The native kernel reads each target patch straight from the
  volume (no patchified copy of the target is ever stored) and writes the loss and d(prediction)
  in the same pass.
"""

from __future__ import annotations

import torch

from ._native import native, use_native
from .patch import patchify_reference


def restore_reference(visible: torch.Tensor, mask_token: torch.Tensor, restore: torch.Tensor) -> torch.Tensor:
    b, n = restore.shape
    pad = mask_token.reshape(1, 1, -1).expand(b, n - visible.shape[1], -1).to(visible.dtype)
    x = torch.cat([visible, pad], dim=1)
    return torch.gather(x, 1, restore.unsqueeze(-1).expand(-1, -1, x.shape[2]))


class _NativeRestore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, visible, mask_token, restore):  # type: ignore[override]
        b, n = restore.shape
        out = torch.empty((b, n, visible.shape[2]), device=visible.device, dtype=visible.dtype)
        tok = mask_token.reshape(-1).to(visible.dtype).contiguous()
        native().mae_restore_fwd(visible.contiguous(), tok, restore.contiguous(), out)
        ctx.save_for_backward(restore)
        ctx.k = visible.shape[1]
        ctx.tok_shape = mask_token.shape
        ctx.tok_dtype = mask_token.dtype
        return out

    @staticmethod
    def backward(ctx, dout):  # type: ignore[override]
        (restore,) = ctx.saved_tensors
        b, n = restore.shape
        dout = dout.contiguous()
        dvis = torch.empty((b, ctx.k, dout.shape[2]), device=dout.device, dtype=dout.dtype)
        dtok = torch.zeros(dout.shape[2], device=dout.device, dtype=torch.float32)
        native().mae_restore_bwd(dout, restore, dvis, dtok)
        return dvis, dtok.reshape(ctx.tok_shape).to(ctx.tok_dtype), None


def restore_with_mask_token(visible: torch.Tensor, mask_token: torch.Tensor, restore: torch.Tensor) -> torch.Tensor:
    if use_native(visible) and visible.dtype == torch.bfloat16:
        return _NativeRestore.apply(visible, mask_token, restore)
    return restore_reference(visible, mask_token, restore)


def norm_pix_mse_reference(
    prediction: torch.Tensor,
    volumes: torch.Tensor,
    mask: torch.Tensor,
    patch: tuple[int, int, int],
    norm_pix: bool = True,
) -> torch.Tensor:
    target = patchify_reference(volumes, patch)
    if norm_pix:
        mean = target.mean(dim=-1, keepdim=True)
        var = target.var(dim=-1, keepdim=True)
        target = (target - mean) / torch.sqrt(var + 1e-6)
    per_patch = (prediction - target).pow(2).mean(dim=-1)
    return (per_patch * mask).sum() / mask.sum().clamp_min(1.0)


class _NativeNormPixMSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, prediction, volumes, mask, patch, norm_pix):  # type: ignore[override]
        pred = prediction.contiguous()
        vol = volumes.contiguous()
        m = mask.float().contiguous()
        loss = torch.zeros((), device=pred.device, dtype=torch.float32)
        grad = torch.empty_like(pred)
        native().norm_pix_mse(pred, vol, m, loss, grad, patch[0], patch[1], patch[2], bool(norm_pix))
        ctx.save_for_backward(grad)
        return loss

    @staticmethod
    def backward(ctx, dloss):  # type: ignore[override]
        (grad,) = ctx.saved_tensors
        return (grad * dloss.to(grad.dtype)), None, None, None, None


def norm_pix_mse(
    prediction: torch.Tensor,
    volumes: torch.Tensor,
    mask: torch.Tensor,
    patch: tuple[int, int, int],
    norm_pix: bool = True,
) -> torch.Tensor:
    if (
        use_native(prediction)
        and prediction.dtype in (torch.bfloat16, torch.float32)
        and volumes.dtype in (torch.float32, torch.bfloat16)
        and patch[2] % 8 == 0
    ):
        return _NativeNormPixMSE.apply(prediction, volumes, mask, tuple(patch), norm_pix)
    return norm_pix_mse_reference(prediction.float(), volumes.float(), mask.float(), patch, norm_pix)


def masked_l1_reference(
    prediction: torch.Tensor,
    volumes: torch.Tensor,
    mask: torch.Tensor,
    patch: tuple[int, ...],
    norm_pix: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """SimMIM's (masked-patch mean L1, visible-patch mean L1) in PyTorch ops."""
    target = patchify_reference(volumes, patch)
    if norm_pix:
        mean = target.mean(dim=-1, keepdim=True)
        var = target.var(dim=-1, keepdim=True)
        target = (target - mean) / torch.sqrt(var + 1e-6)
    per_patch = (prediction.float() - target.float()).abs().mean(dim=-1)
    m = mask.float()
    loss = (per_patch * m).sum() / m.sum().clamp_min(1.0)
    visible = (per_patch * (1 - m)).sum() / (1 - m).sum().clamp_min(1.0)
    return loss, visible.detach()


class _NativeMaskedL1(torch.autograd.Function):
    @staticmethod
    def forward(ctx, prediction, volumes, mask, patch, norm_pix):  # type: ignore[override]
        pred = prediction.contiguous()
        sums = torch.zeros(2, device=pred.device, dtype=torch.float32)
        grad = torch.empty_like(pred)
        native().masked_l1(pred, volumes.contiguous(), mask.float().contiguous(), sums, grad, patch[0], patch[1],
                           patch[2], bool(norm_pix))
        ctx.save_for_backward(grad)
        loss, visible = sums[0].clone(), sums[1].clone()
        ctx.mark_non_differentiable(visible)
        return loss, visible

    @staticmethod
    def backward(ctx, dloss, _dvisible):  # type: ignore[override]
        (grad,) = ctx.saved_tensors
        return grad * dloss.to(grad.dtype), None, None, None, None


def masked_l1(
    prediction: torch.Tensor,
    volumes: torch.Tensor,
    mask: torch.Tensor,
    patch: tuple[int, ...],
    norm_pix: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """(mean L1 over masked patches, mean L1 over visible patches) of (B, N, C * prod(patch)) predictions
    against the patches of (B, C, D, H, W) volumes; the native kernel reads target patches straight
    from the volume and writes d(prediction) in the same pass."""
    if (
        use_native(prediction)
        and len(patch) == 3
        and prediction.dtype in (torch.bfloat16, torch.float32)
        and volumes.dtype in (torch.float32, torch.bfloat16)
        and patch[2] % 8 == 0
    ):
        return _NativeMaskedL1.apply(prediction, volumes, mask, tuple(patch), norm_pix)
    return masked_l1_reference(prediction, volumes, mask, patch, norm_pix)
