"""LayerNorm and RMSNorm on native kernels: one warp-per-row pass in fp32, bf16 in and out.

Forward saves the per-row mean and reciprocal standard deviation; backward recomputes the
normalised row from them and produces dX in the same pass, with the weight and bias gradients
reduced per CTA and summed across CTAs by a second small kernel. `layer_norm_residual` also hands back the
input for a residual branch, so the backward adds that branch's gradient to dX in the same kernel
instead of a separate add. On CPU this is `F.layer_norm`.
Outputs keep the input dtype (the reference's autocast would have produced fp32 and cast again
in the next matmul).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._native import native, use_native
from ._params import grad_sink


class _NativeLayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps, rms):  # type: ignore[override]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y = torch.empty_like(x2)
        rows = x2.shape[0]
        mean = torch.empty(rows, device=x.device, dtype=torch.float32)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        w = weight.float().contiguous() if weight is not None else None
        b = bias.float().contiguous() if bias is not None else None
        native().layernorm_fwd(x2, w, b, y, mean, rstd, float(eps), bool(rms))
        ctx.save_for_backward(x2, w, mean, rstd)
        ctx.sinks = (grad_sink(weight), grad_sink(bias))
        ctx.meta = (shape, weight is not None, bias is not None, rms,
                    weight.dtype if weight is not None else None, bias.dtype if bias is not None else None)
        return y.reshape(shape)

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w, mean, rstd = ctx.saved_tensors
        shape, has_w, has_b, rms, wdtype, bdtype = ctx.meta
        dy2 = dy.reshape(x2.shape).to(x2.dtype).contiguous()
        dx = torch.empty_like(x2)
        n = x2.shape[1]
        w_sink, b_sink = ctx.sinks
        dw = (w_sink if w_sink is not None else torch.zeros(n, device=x2.device, dtype=torch.float32)) if has_w else None
        db = (b_sink if b_sink is not None else torch.zeros(n, device=x2.device, dtype=torch.float32)) if has_b else None
        native().layernorm_bwd(dy2, x2, w, mean, rstd, dx, dw, db, bool(rms), None)
        return (
            dx.reshape(shape),
            dw.to(wdtype) if (dw is not None and w_sink is None) else None,
            db.to(bdtype) if (db is not None and b_sink is None) else None,
            None,
            None,
        )


class _NativeLayerNormResidual(torch.autograd.Function):
    """(LN(x), x): the second output feeds a residual branch; backward returns LN'(dy) + d_residual."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):  # type: ignore[override]
        y = _NativeLayerNorm.forward(ctx, x, weight, bias, eps, False)
        return y, x.view_as(x)

    @staticmethod
    def backward(ctx, dy, dres):  # type: ignore[override]
        x2, w, mean, rstd = ctx.saved_tensors
        shape, has_w, has_b, rms, wdtype, bdtype = ctx.meta
        n = x2.shape[1]
        dy2 = torch.zeros_like(x2) if dy is None else dy.reshape(x2.shape).to(x2.dtype).contiguous()
        dres2 = None if dres is None else dres.reshape(x2.shape).to(x2.dtype).contiguous()
        dx = torch.empty_like(x2)
        w_sink, b_sink = ctx.sinks
        dw = (w_sink if w_sink is not None else torch.zeros(n, device=x2.device, dtype=torch.float32)) if has_w else None
        db = (b_sink if b_sink is not None else torch.zeros(n, device=x2.device, dtype=torch.float32)) if has_b else None
        native().layernorm_bwd(dy2, x2, w, mean, rstd, dx, dw, db, bool(rms), dres2)
        return (
            dx.reshape(shape),
            dw.to(wdtype) if (dw is not None and w_sink is None) else None,
            db.to(bdtype) if (db is not None and b_sink is None) else None,
            None,
        )


def layer_norm_residual(
    x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, eps: float = 1e-5
) -> tuple[torch.Tensor, torch.Tensor]:
    """`(layer_norm(x), x)` for a pre-norm residual block, `h, r = layer_norm_residual(x, ...)`,
    `out = r + f(h)`: both gradients of x are summed inside the LayerNorm backward kernel."""
    if use_native(x) and x.dtype in (torch.bfloat16, torch.float32) and x.shape[-1] % 8 == 0 and x.shape[-1] <= 2048:
        return _NativeLayerNormResidual.apply(x, weight, bias, eps)
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps), x


def layer_norm(
    x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, eps: float = 1e-5
) -> torch.Tensor:
    if use_native(x) and x.dtype in (torch.bfloat16, torch.float32) and x.shape[-1] % 8 == 0 and x.shape[-1] <= 2048:
        return _NativeLayerNorm.apply(x, weight, bias, eps, False)
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float = 1e-6) -> torch.Tensor:
    if use_native(x) and x.dtype in (torch.bfloat16, torch.float32) and x.shape[-1] % 8 == 0 and x.shape[-1] <= 2048:
        return _NativeLayerNorm.apply(x, weight, None, eps, True)
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(x.dtype)
