"""The transformer MLP `residual + fc2(gelu(fc1(x)))` as one autograd node on the native GEMM.

Forward: fc1's epilogue adds the bias, keeps the pre-activation `H` and writes `A = gelu(H)`; fc2's
epilogue adds its bias and the residual. Backward: the `dA = dY @ W2` GEMM multiplies by gelu'(H)
in its epilogue, so `dH` comes out of the tensor cores without a separate elementwise pass;
weight gradients accumulate in fp32. On CPU (or fp32 compute) this is plain PyTorch.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._native import use_native
from ._params import compute_weight, grad_sink
from .linear import ACT_DGELU, ACT_GELU, column_sum, compute_dtype, gemm


class _NativeMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, residual, cdtype):  # type: ignore[override]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(cdtype).contiguous()
        w1c = compute_weight(w1, cdtype).contiguous()
        w2c = compute_weight(w2, cdtype).contiguous()
        b1f = b1.float().contiguous() if b1 is not None else None
        b2f = b2.float().contiguous() if b2 is not None else None
        m = x2.shape[0]
        pre = torch.empty((m, w1.shape[0]), device=x.device, dtype=cdtype)
        act = gemm(x2, w1c, out_dtype=cdtype, bias=b1f, act=ACT_GELU, aux_out=pre)
        res2 = residual.reshape(-1, w2.shape[0]).to(cdtype).contiguous() if residual is not None else None
        y = gemm(act, w2c, out_dtype=cdtype, bias=b2f, residual=res2)
        ctx.save_for_backward(x2, w1c, w2c, pre, act)
        ctx.meta = (shape, b1 is not None, b2 is not None, residual is not None, w1.dtype, w2.dtype)
        ctx.sinks = (grad_sink(w1), grad_sink(b1), grad_sink(w2), grad_sink(b2))
        return y.reshape(*shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w1, w2, pre, act = ctx.saved_tensors
        shape, has_b1, has_b2, has_res, w1dtype, w2dtype = ctx.meta
        sw1, sb1, sw2, sb2 = ctx.sinks
        dy2 = dy.reshape(-1, w2.shape[0]).to(x2.dtype).contiguous()
        dh = gemm(dy2, w2, b_kmajor=False, out_dtype=x2.dtype, act=ACT_DGELU, aux=pre)

        def weight_grad(dout, inp, sink, wshape, wdtype):
            if sink is not None:
                gemm(dout, inp, a_kmajor=False, b_kmajor=False, out=sink.view(wshape), accumulate=True)
                return None
            return gemm(dout, inp, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32).to(wdtype)

        def bias_grad(dout, sink, present, wdtype):
            if not present:
                return None
            if sink is not None:
                column_sum(dout, out=sink, accumulate=True)
                return None
            return column_sum(dout).to(wdtype)

        dw2 = weight_grad(dy2, act, sw2, w2.shape, w2dtype)
        db2 = bias_grad(dy2, sb2, has_b2, w2dtype)
        dx = gemm(dh, w1, b_kmajor=False, out_dtype=x2.dtype).reshape(shape) if ctx.needs_input_grad[0] else None
        dw1 = weight_grad(dh, x2, sw1, w1.shape, w1dtype)
        db1 = bias_grad(dh, sb1, has_b1, w1dtype)
        return dx, dw1, db1, dw2, db2, (dy if has_res else None), None


def mlp(
    x: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor | None,
    w2: torch.Tensor,
    b2: torch.Tensor | None,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    cdtype = compute_dtype(x)
    if cdtype == torch.bfloat16 and use_native(x) and x.shape[-1] % 8 == 0 and w1.shape[0] % 8 == 0 and w2.shape[0] % 8 == 0:
        return _NativeMLP.apply(x, w1, b1, w2, b2, residual, cdtype)
    y = F.linear(F.gelu(F.linear(x, w1, b1)), w2, b2)
    return y if residual is None else residual + y
