"""RMSNorm `x * rsqrt(mean(x^2) + eps) * weight`, computed in fp32 (reference
`src/layers/common/rms_norm.py:13-27`); native kernel on CUDA."""

from __future__ import annotations

import torch
import torch.nn as nn

from ...ops.norm import rms_norm


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def reset_parameters(self) -> None:
        nn.init.ones_(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)
