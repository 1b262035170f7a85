"""DINO / iBOT soft-target cross-entropy and the KoLeo regulariser on native kernels (`csrc/dino_loss.cu`).

`soft_cross_entropy(S, T, pairs, weights, tau, norm)` returns

    (1 / norm) * sum_i sum_j w_ij * ( -sum_k T[pairs_ij, k] * log_softmax(S_i / tau)_k )

in one pass over each student row (log-sum-exp and the pair dot products together) and one pass in
backward; the teacher probabilities get no gradient. `koleo(x, eps)` is
-mean_i log(|| xn_i - xn_nn(i) + eps || + eps) over L2-normalised rows with the nearest neighbour by
dot product, self excluded. Both fall back to the PyTorch formulas (the test oracles) on CPU.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._native import native, use_native


class _SoftCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, S, T, pairs, weights, tau, norm):  # type: ignore[override]
        S = S.contiguous()
        T = T.float().contiguous()
        lse = torch.empty(S.shape[0], device=S.device, dtype=torch.float32)
        loss = torch.empty(S.shape[0], device=S.device, dtype=torch.float32)
        native().soft_ce_fwd(S, T, pairs, weights, float(tau), lse, loss)
        ctx.save_for_backward(S, T, pairs, weights, lse)
        ctx.tau, ctx.norm = float(tau), float(norm)
        return loss.sum() / ctx.norm

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        S, T, pairs, weights, lse = ctx.saved_tensors
        scale = (g.float() / ctx.norm).reshape(1).contiguous()
        dS = torch.empty_like(S)
        native().soft_ce_bwd(S, T, pairs, weights, ctx.tau, lse, scale, dS)
        return dS, None, None, None, None, None


def soft_cross_entropy(S: torch.Tensor, T: torch.Tensor, pairs: torch.Tensor, weights: torch.Tensor, tau: float,
                       norm: float) -> torch.Tensor:
    """S (R, K) student logits, T (Rt, K) teacher probabilities, pairs (R, n) int rows of T, weights (R, n)."""
    if use_native(S) and S.shape[1] % 8 == 0 and pairs.shape[1] <= 4 and S.dtype in (torch.bfloat16, torch.float32):
        return _SoftCE.apply(S, T.detach(), pairs.to(torch.int32).contiguous(), weights.float().contiguous(), tau, norm)
    logp = F.log_softmax(S.float() / tau, dim=-1)
    total = S.new_zeros((), dtype=torch.float32)
    for j in range(pairs.shape[1]):
        total = total - (weights[:, j].float() * (T.detach().float()[pairs[:, j].long()] * logp).sum(-1)).sum()
    return total / norm


class _KoLeo(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps):  # type: ignore[override]
        x = x.float().contiguous()
        b = x.shape[0]
        xn = torch.empty_like(x)
        nn_idx = torch.empty(b, device=x.device, dtype=torch.int32)
        dist = torch.empty(b, device=x.device, dtype=torch.float32)
        loss = torch.empty(1, device=x.device, dtype=torch.float32)
        native().koleo_fwd(x, float(eps), xn, nn_idx, dist, loss)
        ctx.save_for_backward(x, xn, nn_idx, dist)
        ctx.eps = float(eps)
        return loss[0]

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        x, xn, nn_idx, dist = ctx.saved_tensors
        dxn = torch.empty_like(x)
        dx = torch.empty_like(x)
        native().koleo_bwd(x, xn, nn_idx, dist, ctx.eps, g.float().reshape(1).contiguous(), dxn, dx)
        return dx, None


def koleo_reference(x: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    xn = F.normalize(x.float(), eps=eps, p=2, dim=-1)
    dots = xn @ xn.t()
    n = xn.shape[0]
    dots.view(-1)[:: n + 1].fill_(-1)
    nearest = dots.argmax(dim=1)
    d = F.pairwise_distance(xn, xn[nearest], p=2, eps=eps)
    return -torch.log(d + eps).mean()


def koleo(x: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    if use_native(x) and 2 <= x.shape[0] <= 8192 and x.dim() == 2:
        return _KoLeo.apply(x, eps)
    return koleo_reference(x, eps)
