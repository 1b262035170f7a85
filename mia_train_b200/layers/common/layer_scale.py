"""Per-channel LayerScale `x * gamma` (reference `src/layers/common/layer_scale.py:14-31`). Inside
blocks the scale is applied in the output-projection / fc2 GEMM epilogue instead."""

from __future__ import annotations

import torch
import torch.nn as nn


class LayerScale(nn.Module):
    def __init__(self, dim: int, init_values: float = 1e-5, inplace: bool = False, device=None) -> None:
        super().__init__()
        self.inplace = inplace
        self.init_values = init_values
        self.gamma = nn.Parameter(torch.empty(dim, device=device))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.constant_(self.gamma, self.init_values)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x.mul_(self.gamma) if self.inplace else x * self.gamma
