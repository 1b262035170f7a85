"""Rotary position embedding and non-causal attention on native kernels.

Rotation is expressed as a list of channel pairs `(first[p], second[p])` and a per-token angle
table `angles[b, n, p]`; pair p becomes `(x1 cos - x2 sin, x2 cos + x1 sin)`. Both the axial RoPE of
`vit3d`/`muvit3d` (one chunk of the head per spatial axis, reference `src/layers/common/rope.py:41-75`)
and DINOv3's rotate-half RoPE with untouched prefix tokens (reference
`src/layers/dinov3/attention.py:56-67`) are this form: a prefix token simply has angle 0.

Angles are computed by PyTorch from coordinates and the (learnable) inverse frequencies, so
autograd carries `d angles` on to the frequencies; the kernels return `d angles` per token.

`rope_attention(qkv, angles, pairs, scale)` takes the fused projection output (B, N, 3, H, D):
the forward kernel rotates q and k while splitting heads into (B, H, N, D), attention writes
(B, N, H, D) so the output projection reads it without a transpose; the backward runs attention's
backward and then un-rotates dq/dk straight back into the packed (B, N, 3, H, D) gradient.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._native import native, use_native


def rotate_pairs_reference(x: torch.Tensor, angles: torch.Tensor, pairs: torch.Tensor) -> torch.Tensor:
    """x (B, N, H, D); angles (B or 1, N, P); pairs (P, 2) long -> rotated x (fp32 math, x.dtype out)."""
    first, second = pairs[:, 0], pairs[:, 1]
    cos = angles.float().cos().unsqueeze(-2)
    sin = angles.float().sin().unsqueeze(-2)
    x1 = x[..., first].float()
    x2 = x[..., second].float()
    out = x.float().clone()
    out[..., first] = x1 * cos - x2 * sin
    out[..., second] = x2 * cos + x1 * sin
    return out.to(x.dtype)


def attention_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """(B, N, H, D) inputs -> (B, N, H, D) through PyTorch SDPA."""
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=scale)
    return out.transpose(1, 2)


def _native_ok(x: torch.Tensor, head_dim: int) -> bool:
    return x.dtype == torch.bfloat16 and head_dim in (32, 64, 128) and use_native(x)


class _NativeRopeAttention(torch.autograd.Function):
    """Attention (+ RoPE) on the packed projection without splitting it.

    Forward: q and k are rotated into a (B, N, 2, H, D) buffer (skipped without RoPE); the attention
    kernel reads q / k from it and v straight out of `qkv` through strided views. Backward writes dv
    and the rotated-space dk into their slots of the packed gradient, then one kernel un-rotates dq
    and dk in place and reduces the per-token angle gradient.
    """

    @staticmethod
    def forward(ctx, qkv, angles, pairs, scale):  # type: ignore[override]
        b, n, three, h, d = qkv.shape
        qkv = qkv.contiguous()
        ang = angles.float().contiguous() if angles is not None and pairs.numel() else None
        if ang is not None:
            qk = torch.empty((b, n, 2, h, d), device=qkv.device, dtype=qkv.dtype)
            native().rope_qk_fwd(qkv, ang, pairs, qk)
            q, k = qk[:, :, 0], qk[:, :, 1]
        else:
            qk = None
            q, k = qkv[:, :, 0], qkv[:, :, 1]
        v = qkv[:, :, 2]
        o = torch.empty((b, n, h, d), device=qkv.device, dtype=qkv.dtype)
        lse = torch.empty((b, h, n), device=qkv.device, dtype=torch.float32)
        native().attention_fwd_strided(q, k, v, o, lse, float(scale))
        ctx.save_for_backward(qkv, qk, o, lse, ang, pairs)
        ctx.scale = scale
        ctx.angles_shape = angles.shape if angles is not None else None
        ctx.angles_dtype = angles.dtype if angles is not None else None
        return o

    @staticmethod
    def backward(ctx, do):  # type: ignore[override]
        qkv, qk, o, lse, ang, pairs = ctx.saved_tensors
        do = do.to(qkv.dtype).contiguous()
        b, n, _, h, d = qkv.shape
        src = qk if qk is not None else qkv
        q, k, v = src[:, :, 0], src[:, :, 1], qkv[:, :, 2]
        dqkv = torch.empty_like(qkv)
        dang = None
        if ang is not None and ctx.needs_input_grad[1]:
            dang = torch.empty((b, n, pairs.shape[0]), device=qkv.device, dtype=torch.float32)
        native().rope_attention_bwd_packed(q, k, v, o, do, lse, ang, pairs, dqkv, dang, float(ctx.scale))
        if dang is not None:
            if ctx.angles_shape[0] == 1 and b != 1:
                dang = dang.sum(0, keepdim=True)
            dang = dang.to(ctx.angles_dtype)
        return dqkv, dang, None, None


def rope_attention(
    qkv: torch.Tensor, angles: torch.Tensor | None, pairs: torch.Tensor | None, scale: float
) -> torch.Tensor:
    """Packed (B, N, 3, H, D) projections -> attention output (B, N, H, D)."""
    if _native_ok(qkv, qkv.shape[-1]):
        if pairs is None:
            pairs = torch.zeros((0, 2), dtype=torch.int32, device=qkv.device)
        return _NativeRopeAttention.apply(qkv, angles, pairs.to(device=qkv.device, dtype=torch.int32), scale)
    q, k, v = qkv.unbind(dim=2)
    if angles is not None and pairs is not None and pairs.numel():
        p = pairs.long().to(qkv.device)
        q = rotate_pairs_reference(q, angles, p)
        k = rotate_pairs_reference(k, angles, p)
    return attention_reference(q, k, v, scale)


class _NativeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale):  # type: ignore[override]
        qh = q.transpose(1, 2).contiguous()
        kh = k.transpose(1, 2).contiguous()
        vh = v.transpose(1, 2).contiguous()
        b, h, n, d = qh.shape
        o = torch.empty((b, n, h, d), device=q.device, dtype=q.dtype)
        lse = torch.empty((b, h, n), device=q.device, dtype=torch.float32)
        native().attention_fwd(qh, kh, vh, o, lse, float(scale))
        ctx.save_for_backward(qh, kh, vh, o, lse)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):  # type: ignore[override]
        qh, kh, vh, o, lse = ctx.saved_tensors
        do = do.to(qh.dtype).contiguous()
        dq = torch.empty_like(qh)
        dk = torch.empty_like(kh)
        dv = torch.empty_like(vh)
        native().attention_bwd(qh, kh, vh, o, do, lse, dq, dk, dv, float(ctx.scale))
        return dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2), None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """(B, Nq, H, D), (B, Nk, H, D), (B, Nk, H, D) -> (B, Nq, H, D)."""
    if _native_ok(q, q.shape[-1]) and k.dtype == q.dtype and v.dtype == q.dtype:
        return _NativeAttention.apply(q, k, v, scale)
    return attention_reference(q, k, v, scale)


def rotate_pairs(x: torch.Tensor, angles: torch.Tensor, pairs: torch.Tensor) -> torch.Tensor:
    """Rotate (B, N, H, D) by per-token angles; autograd flows to x and angles (PyTorch math)."""
    return rotate_pairs_reference(x, angles, pairs.long().to(x.device))
