"""Linear layers on the hand-written tcgen05 GEMM, with fused epilogues.

`linear(x, weight, bias, activation, residual, gamma)` computes

    y = residual + gamma * act(x @ weight.T + bias)

where every term but the product is optional. On CUDA with bf16 compute (bf16 inputs or a bf16
autocast region) it runs `_C.gemm`, whose epilogue applies bias, GELU, LayerScale and the residual
add while the accumulator is still in tensor memory. With `activation="gelu"` the pre-activation is
kept for the backward pass, whose `dX` GEMM of the next layer fuses the GELU derivative.

Backward: dX = dY @ W runs with W read N-major, dW = dY^T @ X with both operands read M-major (no
transposes are materialised), accumulating directly into an fp32 gradient; the bias gradient is a
column-sum kernel. fp32 compute on CUDA (precision = "fp32") uses PyTorch's matmul: the native
kernels are bf16-only.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ._native import native, use_native
from ._params import compute_weight, grad_sink

ACT_NONE, ACT_GELU, ACT_DGELU = 0, 1, 2
_ACTS = {None: ACT_NONE, "none": ACT_NONE, "gelu": ACT_GELU}


def compute_dtype(x: torch.Tensor) -> torch.dtype:
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    if not x.is_cuda and torch.is_autocast_enabled("cpu"):
        return torch.get_autocast_dtype("cpu")
    return x.dtype


def gelu_reference(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x)


def gelu_grad_reference(h: torch.Tensor) -> torch.Tensor:
    """d gelu(h) / dh for the exact (erf) GELU."""
    h = h.float()
    cdf = 0.5 * (1.0 + torch.erf(h / math.sqrt(2.0)))
    pdf = torch.exp(-0.5 * h * h) / math.sqrt(2.0 * math.pi)
    return cdf + h * pdf


# When a list, every `gemm` call appends (M, N, K, layout, out dtype, act, accumulate, residual): the
# per-shape profile in ops/microbench.py pairs these with the kernels' device times.
GEMM_TRACE: list | None = None


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_kmajor: bool = True,
    b_kmajor: bool = True,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    aux: torch.Tensor | None = None,
    gamma: torch.Tensor | None = None,
    act: int = ACT_NONE,
    accumulate: bool = False,
    aux_out: torch.Tensor | None = None,
    colsum: torch.Tensor | None = None,
    colsum_scale: float = 1.0,
    a2: torch.Tensor | None = None,
    b2: torch.Tensor | None = None,
) -> torch.Tensor:
    """D[M, N] = sum_k A[m, k] B[n, k] with epilogue; operands given in their physical layout.

    `a` is (M, K) when `a_kmajor` else (K, M); `b` is (N, K) when `b_kmajor` else (K, N).
    Epilogue order: acc (+ bias[n]) -> act -> (* gamma[n]) -> (+ residual[m, n]) -> (+ out if
    accumulate). `act=ACT_GELU` writes the pre-activation to `aux_out` when given;
    `act=ACT_DGELU` multiplies by gelu'(aux[m, n]). `colsum` (fp32, N) receives
    `+= sum_m exp(acc[m, n] * colsum_scale)` computed from the accumulator in the same epilogue.
    `a2` (M, K2) and `b2` (N, K2), both K-major, add `a2 @ b2.T` to the accumulator before the
    epilogue (the K loop continues over them).
    """
    m = a.shape[0] if a_kmajor else a.shape[1]
    n = b.shape[0] if b_kmajor else b.shape[1]
    if GEMM_TRACE is not None:
        k = a.shape[1] if a_kmajor else a.shape[0]
        GEMM_TRACE.append((m, n, k, ("n" if a_kmajor else "t") + ("n" if b_kmajor else "t"),
                           "f32" if (out is not None and out.dtype == torch.float32) or out_dtype == torch.float32 else "bf16",
                           act, accumulate, residual is not None))
    if out is None:
        out = torch.empty((m, n), device=a.device, dtype=out_dtype)
    if use_native(a):
        native().gemm(a, b, out, bias, residual, aux, gamma, aux_out, a_kmajor, b_kmajor, act, accumulate, colsum,
                      float(colsum_scale), a2, b2)
        return out
    am = a if a_kmajor else a.t()
    bm = b if b_kmajor else b.t()
    acc = am.float() @ bm.float().t()
    if a2 is not None:
        acc = acc + a2.float() @ b2.float().t()
    if bias is not None:
        acc = acc + bias.float()
    if act == ACT_GELU:
        if aux_out is not None:
            aux_out.copy_(acc)
        acc = gelu_reference(acc)
    elif act == ACT_DGELU:
        acc = acc * gelu_grad_reference(aux)
    if gamma is not None:
        acc = acc * gamma.float()
    if residual is not None:
        acc = acc + residual.float()
    if accumulate:
        acc = acc + out.float()
    if colsum is not None:
        colsum.add_(torch.exp(acc * colsum_scale).sum(0))
    out.copy_(acc)
    return out


def column_sum(x: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """fp32 sum over rows of a (M, N) matrix -> (N,)."""
    if out is None:
        out = torch.zeros(x.shape[1], device=x.device, dtype=torch.float32)
        accumulate = False
    if use_native(x):
        native().column_sum(x, out, accumulate)
        return out
    s = x.float().sum(0)
    out.copy_(out + s if accumulate else s)
    return out


class _NativeLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, residual, gamma, act, cdtype):  # type: ignore[override]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.dtype != cdtype:
            x2 = x2.to(cdtype)
        x2 = x2.contiguous()
        w = compute_weight(weight, cdtype).reshape(weight.shape[0], -1).contiguous()
        res2 = None
        if residual is not None:
            res2 = residual.reshape(-1, weight.shape[0])
            if res2.dtype != cdtype:
                res2 = res2.to(cdtype)
            res2 = res2.contiguous()
        pre = torch.empty((x2.shape[0], weight.shape[0]), device=x.device, dtype=cdtype) if act == ACT_GELU else None
        g = gamma.to(torch.float32).contiguous() if gamma is not None else None
        bf = bias.to(torch.float32).contiguous() if bias is not None else None
        y = gemm(x2, w, out_dtype=cdtype, bias=bf, residual=res2, gamma=g, act=act, aux_out=pre)
        ctx.save_for_backward(x2, w, pre, g, bf)
        ctx.meta = (shape, act, bias is not None, residual is not None, gamma is not None, weight.dtype)
        ctx.weight_shape = weight.shape
        ctx.sinks = (grad_sink(weight), grad_sink(bias))
        return y.reshape(*shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w, pre, g, bf = ctx.saved_tensors
        shape, act, has_bias, has_res, has_gamma, wdtype = ctx.meta
        n = w.shape[0]
        dy2 = dy.reshape(-1, n)
        if dy2.dtype != x2.dtype:
            dy2 = dy2.to(x2.dtype)
        dy2 = dy2.contiguous()
        dres = dy if has_res else None
        dgamma = None
        dz = dy2
        if has_gamma:
            # d(gamma * h)/dgamma needs h = act(xW^T + b); recompute it once (cheap next to the GEMMs).
            h = gemm(x2, w, out_dtype=torch.float32, bias=bf, act=act)
            dgamma = (dy2.float() * h).sum(0).to(wdtype)
            dz = (dy2.float() * g).to(x2.dtype)
        if act == ACT_GELU:
            dz = (dz.float() * gelu_grad_reference(pre)).to(x2.dtype).contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dz, w, b_kmajor=False, out_dtype=x2.dtype).reshape(shape)
        w_sink, b_sink = ctx.sinks
        dw = None
        if ctx.needs_input_grad[1]:
            if w_sink is not None:
                gemm(dz, x2, a_kmajor=False, b_kmajor=False, out=w_sink.view(w.shape), accumulate=True)
            else:
                dw = gemm(dz, x2, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32)
                dw = dw.to(wdtype).view(ctx.weight_shape)
        db = None
        if has_bias and ctx.needs_input_grad[2]:
            if b_sink is not None:
                column_sum(dz, out=b_sink, accumulate=True)
            else:
                db = column_sum(dz).to(wdtype)
        return dx, dw, db, dres, dgamma, None, None


def linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
    residual: torch.Tensor | None = None,
    gamma: torch.Tensor | None = None,
) -> torch.Tensor:
    """`residual + gamma * act(x @ weight.T + bias)`; see the module docstring.

    `weight` may have more than two dims (a kernel == stride convolution's weight): its trailing
    dims are flattened, in the convolution's own order.
    """
    act = _ACTS[activation]
    cdtype = compute_dtype(x)
    if cdtype == torch.bfloat16 and use_native(x) and x.shape[-1] % 8 == 0 and weight.shape[0] % 8 == 0:
        return _NativeLinear.apply(x, weight, bias, residual, gamma, act, cdtype)
    y = F.linear(x, weight.reshape(weight.shape[0], -1), bias)
    if act == ACT_GELU:
        y = F.gelu(y)
    if gamma is not None:
        y = y * gamma
    if residual is not None:
        y = residual + y
    return y


class _NativeLoRALinear(torch.autograd.Function):
    """`act(x W^T + b + s (x A^T) B^T)` with the low-rank delta accumulated into the base GEMM's tile.

    Forward: h = x A^T (rank r), then one GEMM whose K loop runs over x / W and then over h / (s B)
    into the same tensor-memory accumulator, with bias and GELU in the epilogue. Backward:
    dZ = dY (* gelu'), t = dZ (s B); dX = dZ W + t A (the second GEMM accumulates into dX),
    dA = t^T x, dB = s dZ^T h, dW = dZ^T x (when the base weight trains), db = column sums of dZ.
    """

    @staticmethod
    def forward(ctx, x, weight, bias, lora_a, lora_b, scaling, residual, act, cdtype):  # type: ignore[override]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(cdtype).contiguous()
        w = compute_weight(weight, cdtype).contiguous()
        a = lora_a.to(cdtype).contiguous()
        s = float(scaling)
        bs = (lora_b.float() * s).to(cdtype).contiguous()
        h = gemm(x2, a, out_dtype=cdtype)
        res2 = residual.reshape(-1, w.shape[0]).to(cdtype).contiguous() if residual is not None else None
        pre = torch.empty((x2.shape[0], w.shape[0]), device=x.device, dtype=cdtype) if act == ACT_GELU else None
        bf = bias.float().contiguous() if bias is not None else None
        y = gemm(x2, w, out_dtype=cdtype, bias=bf, act=act, aux_out=pre, residual=res2, a2=h, b2=bs)
        ctx.save_for_backward(x2, w, a, bs, h, pre)
        ctx.meta = (shape, act, bias is not None, residual is not None, s, weight.dtype, lora_a.dtype, lora_b.dtype,
                    bias.dtype if bias is not None else None)
        ctx.sinks = (grad_sink(weight), grad_sink(bias))
        return y.reshape(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w, a, bs, h, pre = ctx.saved_tensors
        shape, act, has_b, has_res, s, wdt, adt, bdt, biasdt = ctx.meta
        n = w.shape[0]
        dz = dy.reshape(-1, n).to(x2.dtype).contiguous()
        if act == ACT_GELU:
            dz = (dz.float() * gelu_grad_reference(pre)).to(x2.dtype).contiguous()
        t = gemm(dz, bs, b_kmajor=False, out_dtype=x2.dtype)  # (M, r) = dZ (s B)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dz, w, b_kmajor=False, out_dtype=x2.dtype)
            gemm(t, a, b_kmajor=False, out=dx, accumulate=True)
            dx = dx.reshape(shape)
        da = gemm(t, x2, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32).to(adt)
        db_lora = (gemm(dz, h, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32) * s).to(bdt)
        w_sink, b_sink = ctx.sinks
        dw = None
        if ctx.needs_input_grad[1]:
            if w_sink is not None:
                gemm(dz, x2, a_kmajor=False, b_kmajor=False, out=w_sink.view(w.shape), accumulate=True)
            else:
                dw = gemm(dz, x2, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32).to(wdt)
        dbias = None
        if has_b and ctx.needs_input_grad[2]:
            if b_sink is not None:
                column_sum(dz, out=b_sink, accumulate=True)
            else:
                dbias = column_sum(dz).to(biasdt)
        return dx, dw, dbias, da, db_lora, None, (dy if has_res else None), None, None


def lora_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    lora_a: torch.Tensor,
    lora_b: torch.Tensor,
    scaling: float,
    activation: str | None = None,
    residual: torch.Tensor | None = None,
) -> torch.Tensor | None:
    """`residual + act(x W^T + b + scaling (x A^T) B^T)` on one native GEMM, or None when the native
    path does not apply (the caller then composes it from separate ops)."""
    act = _ACTS[activation]
    cdtype = compute_dtype(x)
    r = lora_a.shape[0]
    if not (cdtype == torch.bfloat16 and use_native(x) and x.shape[-1] % 8 == 0 and weight.shape[0] % 8 == 0
            and r % 8 == 0 and weight.dim() == 2):
        return None
    return _NativeLoRALinear.apply(x, weight, bias, lora_a, lora_b, float(scaling), residual, act, cdtype)

