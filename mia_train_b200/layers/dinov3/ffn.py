"""DINOv3 feed-forward layers (reference `src/layers/dinov3/ffn.py:19-91`).

`Mlp` (fc1 -> GELU -> fc2) and `SwiGLUFFN` (w3(silu(w1 x) * w2 x), hidden = ceil(2/3 h) aligned),
with `forward_list` over concatenated crops. `forward(x, residual=, gamma=)` fuses the block's
LayerScale and residual add into the last projection's epilogue; `Mlp` runs fc1+GELU+fc2 as one
native MLP node when neither projection is LoRA-adapted.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.nn as nn
import torch.nn.functional as F

from ...ops.mlp import mlp
from ..common.batched_tokens import cat_keep_shapes, uncat_with_shapes
from ..common.lora import apply_linear, needs_per_layer


class ListForwardMixin:
    def forward(self, x: torch.Tensor, residual=None, gamma=None) -> torch.Tensor:  # pragma: no cover
        raise NotImplementedError

    def forward_list(self, x_list: list[torch.Tensor], residual_list=None, gamma=None) -> list[torch.Tensor]:
        flat, shapes, counts = cat_keep_shapes(x_list)
        res = cat_keep_shapes(residual_list)[0] if residual_list is not None else None
        return uncat_with_shapes(self.forward(flat, residual=res, gamma=gamma), shapes, counts)


class Mlp(nn.Module, ListForwardMixin):
    def __init__(
        self,
        in_features: int,
        hidden_features: int | None = None,
        out_features: int | None = None,
        act_layer: Callable[..., nn.Module] = nn.GELU,
        drop: float = 0.0,
        bias: bool = True,
        device=None,
    ) -> None:
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features, bias=bias, device=device)
        self.act = act_layer()
        self.fc2 = nn.Linear(hidden_features, out_features, bias=bias, device=device)
        self.drop = nn.Dropout(drop)

    def forward(self, x: torch.Tensor, residual=None, gamma=None) -> torch.Tensor:
        if self.training and self.drop.p > 0:  # dropout between the layers: unfused
            y = self.drop(apply_linear(self.fc2, self.drop(self.act(apply_linear(self.fc1, x)))))
            if gamma is not None:
                y = y * gamma
            return y if residual is None else residual + y
        exact_gelu = isinstance(self.act, nn.GELU) and getattr(self.act, "approximate", "none") == "none"
        if exact_gelu and gamma is None and not (needs_per_layer(self.fc1) or needs_per_layer(self.fc2)):
            return mlp(x, self.fc1.weight, self.fc1.bias, self.fc2.weight, self.fc2.bias, residual=residual)
        h = apply_linear(self.fc1, x, activation="gelu") if exact_gelu else self.act(apply_linear(self.fc1, x))
        return apply_linear(self.fc2, h, residual=residual, gamma=gamma)


class SwiGLUFFN(nn.Module, ListForwardMixin):
    def __init__(
        self,
        in_features: int,
        hidden_features: int | None = None,
        out_features: int | None = None,
        act_layer: Callable[..., nn.Module] | None = None,
        drop: float = 0.0,
        bias: bool = True,
        align_to: int = 8,
        device=None,
    ) -> None:
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        d = int(hidden_features * 2 / 3)
        hidden = d + (-d % align_to)
        self.w1 = nn.Linear(in_features, hidden, bias=bias, device=device)
        self.w2 = nn.Linear(in_features, hidden, bias=bias, device=device)
        self.w3 = nn.Linear(hidden, out_features, bias=bias, device=device)

    def forward(self, x: torch.Tensor, residual=None, gamma=None) -> torch.Tensor:
        hidden = F.silu(apply_linear(self.w1, x)) * apply_linear(self.w2, x)
        return apply_linear(self.w3, hidden, residual=residual, gamma=gamma)
