"""DINO / iBOT projection head (reference `src/layers/dinov3/head.py:22-89`).

MLP `in -> hidden (GELU) -> ... -> bottleneck`, L2 normalisation, then a bias-free prototype layer
`last_layer` (bottleneck -> n_prototypes). Parameter names match the reference (`mlp.0`, `mlp.2`,
... , `last_layer`).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.nn.init import trunc_normal_

from ...ops.linear import linear


class DINOHead(nn.Module):
    def __init__(
        self,
        in_dim: int,
        out_dim: int,
        use_bn: bool = False,
        nlayers: int = 3,
        hidden_dim: int = 2048,
        bottleneck_dim: int = 256,
        mlp_bias: bool = True,
    ) -> None:
        super().__init__()
        nlayers = max(nlayers, 1)
        self.mlp = _build_mlp(nlayers, in_dim, bottleneck_dim, hidden_dim=hidden_dim, use_bn=use_bn, bias=mlp_bias)
        self.last_layer = nn.Linear(bottleneck_dim, out_dim, bias=False)

    def init_weights(self) -> None:
        self.apply(_init_weights)

    def forward_mlp(self, x: torch.Tensor) -> torch.Tensor:
        """The MLP on the native GEMM, with GELU fused into each hidden layer's epilogue."""
        layers = list(self.mlp) if isinstance(self.mlp, nn.Sequential) else [self.mlp]
        i = 0
        while i < len(layers):
            layer = layers[i]
            nxt = layers[i + 1] if i + 1 < len(layers) else None
            if isinstance(layer, nn.Linear) and isinstance(nxt, nn.GELU):
                x = linear(x, layer.weight, layer.bias, activation="gelu")
                i += 2
            elif isinstance(layer, nn.Linear):
                x = linear(x, layer.weight, layer.bias)
                i += 1
            else:
                x = layer(x)
                i += 1
        return x

    def forward(self, x: torch.Tensor, exp_colsum: torch.Tensor | None = None, temperature: float | None = None):
        """Prototype logits. With `exp_colsum` (fp32, n_prototypes; no autograd -- the teacher's use)
        the prototype GEMM also adds sum_b exp(logit[b, k] / temperature) into it from its epilogue:
        the first column reduction of Sinkhorn-Knopp centring, without another pass over the logits."""
        x = self.forward_mlp(x)
        eps = 1e-6 if x.dtype == torch.float16 else 1e-12
        x = F.normalize(x, dim=-1, p=2, eps=eps)
        if exp_colsum is None:
            return linear(x, self.last_layer.weight)
        from ...ops._native import use_native
        from ...ops.linear import compute_dtype, gemm

        cdtype = compute_dtype(x)
        w = self.last_layer.weight
        if cdtype == torch.bfloat16 and use_native(x) and x.shape[-1] % 8 == 0 and w.shape[0] % 8 == 0:
            x2 = x.reshape(-1, x.shape[-1]).to(cdtype).contiguous()
            out = gemm(x2, w.to(cdtype).contiguous(), out_dtype=torch.float32, colsum=exp_colsum,
                       colsum_scale=1.0 / float(temperature))
            return out.reshape(*x.shape[:-1], w.shape[0])
        logits = linear(x, w)
        exp_colsum.add_(torch.exp(logits.float().reshape(-1, w.shape[0]) / float(temperature)).sum(0))
        return logits


def _init_weights(module: nn.Module) -> None:
    if isinstance(module, nn.Linear):
        trunc_normal_(module.weight, std=0.02)
        if module.bias is not None:
            nn.init.zeros_(module.bias)


def _build_mlp(nlayers, in_dim, bottleneck_dim, hidden_dim=None, use_bn=False, bias=True) -> nn.Module:
    if nlayers == 1:
        return nn.Linear(in_dim, bottleneck_dim, bias=bias)
    if hidden_dim is None:
        raise ValueError("hidden_dim is required when nlayers > 1")
    layers: list[nn.Module] = [nn.Linear(in_dim, hidden_dim, bias=bias)]
    if use_bn:
        layers.append(nn.BatchNorm1d(hidden_dim))
    layers.append(nn.GELU())
    for _ in range(nlayers - 2):
        layers.append(nn.Linear(hidden_dim, hidden_dim, bias=bias))
        if use_bn:
            layers.append(nn.BatchNorm1d(hidden_dim))
        layers.append(nn.GELU())
    layers.append(nn.Linear(hidden_dim, bottleneck_dim, bias=bias))
    return nn.Sequential(*layers)
