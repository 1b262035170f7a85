"""Pre-norm transformer block positioned by axial RoPE (reference `src/layers/common/blocks.py:19-47`).

`x + attn(LN(x), rope=rotary(coords))`, then `x + mlp(LN(x))` with a GELU MLP; each block owns its
rotary frequencies. Parameter names match the reference (`norm1`, `attn`, `rotary`, `norm2`,
`mlp.0`, `mlp.2`). The residual adds are fused into the epilogues of the output-projection and fc2
GEMMs, and fc1+GELU+fc2 run as one native MLP node.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ...ops.mlp import mlp
from ...ops.norm import layer_norm, layer_norm_residual
from .attention import SelfAttention
from .lora import apply_linear, needs_per_layer
from .rope import AxialRotaryEmbedding


class TransformerBlock(nn.Module):
    def __init__(
        self,
        dim: int,
        num_heads: int,
        mlp_ratio: float = 4.0,
        attention_backend: str = "auto",
        spatial_rank: int = 3,
        rotary_base: float = 10000.0,
        rotary: bool = True,
    ) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(dim)
        self.attn = SelfAttention(dim, num_heads, backend=attention_backend)
        self.rotary = AxialRotaryEmbedding(dim // num_heads, spatial_rank, base=rotary_base) if rotary else None
        self.norm2 = nn.LayerNorm(dim)
        hidden = int(dim * mlp_ratio)
        self.mlp = nn.Sequential(nn.Linear(dim, hidden), nn.GELU(), nn.Linear(hidden, dim))

    def forward(self, x: torch.Tensor, coords: torch.Tensor | None = None) -> torch.Tensor:
        rope = self.rotary(coords) if (self.rotary is not None and coords is not None) else None
        h, r = layer_norm_residual(x, self.norm1.weight, self.norm1.bias, self.norm1.eps)
        x = self.attn(h, rope=rope, residual=r)
        h, r = layer_norm_residual(x, self.norm2.weight, self.norm2.bias, self.norm2.eps)
        fc1, fc2 = self.mlp[0], self.mlp[2]
        if needs_per_layer(fc1) or needs_per_layer(fc2):
            return apply_linear(fc2, apply_linear(fc1, h, activation="gelu"), residual=r)
        return mlp(h, fc1.weight, fc1.bias, fc2.weight, fc2.bias, residual=r)
