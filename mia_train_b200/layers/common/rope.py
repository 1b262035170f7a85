"""Axial rotary position embedding over continuous per-token coordinates.

Same parameterisation as the reference's `src/layers/common/rope.py:23-120`: the head dimension is
split into one even-width chunk per spatial axis (remainder to the first axis), each axis has its
own learnable inverse frequencies initialised to `base ** (-2i / width)`, angles are computed in
fp32, and each chunk is rotated half-against-half by its axis coordinate. Parameter names
(`inv_freqs.{axis}`) match the reference's so checkpoints load.

The embedding returns `RotaryTables`: the angle table `(B, N, P)` plus the channel pairs it
rotates. Attention hands both to the native fused rope+attention kernel; calling the tables on a
(B, N, H, D) tensor rotates it in PyTorch, as the reference's callable does.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from ...ops._native import native, use_native
from ...ops._params import grad_sink
from ...ops.attention import rotate_pairs


def split_rope_dims(head_dim: int, spatial_rank: int) -> tuple[int, ...]:
    if head_dim < 2 * spatial_rank:
        raise ValueError(
            f"head_dim {head_dim} cannot cover {spatial_rank} spatial axes: each axis needs at least "
            f"one channel pair, so head_dim must be at least {2 * spatial_rank}"
        )
    each = 2 * (head_dim // spatial_rank // 2)
    dims = [each] * spatial_rank
    dims[0] += 2 * ((head_dim - sum(dims)) // 2)
    return tuple(dims)


def axial_pairs(axis_dims: tuple[int, ...]) -> torch.Tensor:
    """(P, 2) channel pairs: within each axis chunk, channel j rotates with channel j + width/2."""
    pairs = []
    start = 0
    for width in axis_dims:
        half = width // 2
        pairs.extend((start + j, start + half + j) for j in range(half))
        start += width
    return torch.tensor(pairs, dtype=torch.int32).reshape(-1, 2)


@dataclass(frozen=True)
class RotaryTables:
    """Per-token rotation angles (B, N, P) fp32 and the channel pairs they apply to."""

    angles: torch.Tensor
    pairs: torch.Tensor

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return rotate_pairs(x, self.angles, self.pairs)


class _AxialAngles(torch.autograd.Function):
    """Native angle table; frequency gradients are added straight into `main_grad` when present."""

    @staticmethod
    def forward(ctx, coords, *freqs):  # type: ignore[override]
        coords = coords.float().contiguous()
        ctx.save_for_backward(coords, *freqs)
        return native().axial_angles_fwd(coords, [f.contiguous() for f in freqs])

    @staticmethod
    def backward(ctx, dangles):  # type: ignore[override]
        coords, *freqs = ctx.saved_tensors
        sinks = [grad_sink(f) for f in freqs]
        outs = [s if s is not None else torch.zeros_like(f) for s, f in zip(sinks, freqs, strict=True)]
        native().axial_angles_bwd(dangles.float().contiguous(), coords, [f.contiguous() for f in freqs], outs)
        grads = [None if s is not None else o for s, o in zip(sinks, outs, strict=True)]
        return (None, *grads)


class AxialRotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, spatial_rank: int, base: float = 10000.0) -> None:
        super().__init__()
        if base <= 1.0:
            raise ValueError(f"rotary base must be greater than 1, got {base}")
        self.axis_dims = split_rope_dims(head_dim, spatial_rank)
        self.spatial_rank = spatial_rank
        self.inv_freqs = nn.ParameterList(
            nn.Parameter(1.0 / (base ** (torch.arange(0, w, 2).float() / w))) for w in self.axis_dims
        )
        self.register_buffer("pairs", axial_pairs(self.axis_dims), persistent=False)

    @property
    def rotary_dim(self) -> int:
        return sum(self.axis_dims)

    def angles(self, coords: torch.Tensor) -> torch.Tensor:
        """(B, N, rank) coordinates -> (B, N, P) fp32 angles, axis chunks concatenated."""
        if coords.shape[-1] != self.spatial_rank:
            raise ValueError(
                f"expected coordinates with {self.spatial_rank} components on the last axis, got "
                f"{tuple(coords.shape)}"
            )
        freqs = list(self.inv_freqs)
        if coords.is_cuda and all(type(f) is nn.Parameter or type(f) is torch.Tensor for f in freqs) and use_native(coords):
            return _AxialAngles.apply(coords, *freqs)
        per_axis = [
            coords[..., a].float().unsqueeze(-1) * f.float() for a, f in enumerate(self.inv_freqs)
        ]
        return torch.cat(per_axis, dim=-1)

    def forward(self, coords: torch.Tensor) -> RotaryTables:
        return RotaryTables(self.angles(coords), self.pairs)
