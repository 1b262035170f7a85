"""DINOv3 rotary position embeddings: 2D, 3D and 3D "superposition" (reference
`src/layers/dinov3/rope.py:27-474`).

Same buffers (`periods`, `depth_periods`), parameter (`depth_scale`), coordinate normalisation
(`min` / `max` / `separate`, then mapped to [-1, 1]) and train-time augmentation (`shift_coords`,
`jitter_coords`, `rescale_coords`) as the reference, so released checkpoints load and the tables
agree. The forward returns `RopeTables`: a `(sin, cos)` pair exactly like the reference's (each
(HW, D_head), angles tiled twice) that also carries the untiled angles (HW, D_head // 2). The
native attention consumes the angles directly as channel pairs (i, i + D_head / 2), which is what
`rope_rotate_half` applies.
"""

from __future__ import annotations

import math
from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F

NORMALIZE = ("min", "max", "separate")


class RopeTables:
    """`.angles` of shape (HW, D_head // 2), and the `(sin, cos)` pair of shape (HW, D_head) (angles
    tiled twice) when unpacked or indexed like the reference's tuple; the pair is computed on first
    use (the native attention only needs the angles).

    Not a tuple on purpose: FSDP rebuilds tuple forward arguments element by element (and may cast
    them), which would lose the angles; an object of this class passes through untouched."""

    __slots__ = ("angles", "_pair")

    def __init__(self, angles: torch.Tensor) -> None:
        self.angles = angles
        self._pair: tuple[torch.Tensor, torch.Tensor] | None = None

    def _tables(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self._pair is None:
            tiled = self.angles.tile(2)
            self._pair = (torch.sin(tiled), torch.cos(tiled))
        return self._pair

    def __iter__(self):
        return iter(self._tables())

    def __getitem__(self, i: int) -> torch.Tensor:
        return self._tables()[i]

    def __len__(self) -> int:
        return 2


def _axis_coords(sizes: tuple[int, ...], mode: str, dtype, device) -> list[torch.Tensor]:
    if mode not in NORMALIZE:
        raise ValueError(f"Unknown normalize_coords: {mode}")
    if mode == "max":
        denom = [max(sizes)] * len(sizes)
    elif mode == "min":
        denom = [min(sizes)] * len(sizes)
    else:
        denom = list(sizes)
    return [torch.arange(0.5, s, dtype=dtype, device=device) / d for s, d in zip(sizes, denom, strict=True)]


def _augment(coords: torch.Tensor, module: nn.Module, per_axis: int) -> torch.Tensor:
    """Train-time shift / jitter / rescale of (N, per_axis) coordinates (reference order)."""
    dd = {"dtype": coords.dtype, "device": coords.device}
    if module.training and module.shift_coords is not None:
        coords = coords + torch.empty(per_axis, **dd).uniform_(-module.shift_coords, module.shift_coords)[None]
    if module.training and module.jitter_coords is not None:
        jmax = math.log(module.jitter_coords)
        coords = coords * torch.empty(per_axis, **dd).uniform_(-jmax, jmax).exp()[None]
    if module.training and module.rescale_coords is not None:
        rmax = math.log(module.rescale_coords)
        coords = coords * torch.empty(1, **dd).uniform_(-rmax, rmax).exp()
    return coords


def _geometric_periods(count: int, denom: int, base: float | None, min_period, max_period, dtype, device):
    if base is not None:
        return base ** (2 * torch.arange(count, dtype=dtype, device=device) / denom)
    ratio = max_period / min_period
    periods = ratio ** torch.linspace(0, 1, count, dtype=dtype, device=device)
    return periods / ratio * max_period


class _RopeBase(nn.Module):
    def _common_init(
        self, embed_dim, num_heads, base, min_period, max_period, normalize_coords, shift_coords, jitter_coords,
        rescale_coords, dtype,
    ) -> None:
        both = min_period is not None and max_period is not None
        if (base is None and not both) or (base is not None and both):
            raise ValueError("Either `base` or `min_period`+`max_period` must be provided.")
        self.base = base
        self.min_period = min_period
        self.max_period = max_period
        self.D_head = embed_dim // num_heads
        self.normalize_coords = normalize_coords
        self.shift_coords = shift_coords
        self.jitter_coords = jitter_coords
        self.rescale_coords = rescale_coords
        self.dtype = dtype


class RopePositionEmbedding(_RopeBase):
    """2D: `periods` (D_head // 4); angles = 2 pi coord / period per axis, (HW, D_head // 2)."""

    periods: torch.Tensor

    def __init__(
        self,
        embed_dim: int,
        *,
        num_heads: int,
        base: float | None = 100.0,
        min_period: float | None = None,
        max_period: float | None = None,
        normalize_coords: Literal["min", "max", "separate"] = "separate",
        shift_coords: float | None = None,
        jitter_coords: float | None = None,
        rescale_coords: float | None = None,
        dtype: torch.dtype | None = None,
        device: torch.device | None = None,
    ) -> None:
        super().__init__()
        assert embed_dim % (4 * num_heads) == 0
        self._common_init(embed_dim, num_heads, base, min_period, max_period, normalize_coords, shift_coords,
                          jitter_coords, rescale_coords, dtype)
        self.register_buffer("periods", torch.empty(self.D_head // 4, device=device, dtype=dtype), persistent=True)
        self._init_weights()

    def angles(self, *, H: int, W: int) -> torch.Tensor:
        ch, cw = _axis_coords((H, W), self.normalize_coords, self.dtype, self.periods.device)
        coords = torch.stack(torch.meshgrid(ch, cw, indexing="ij"), dim=-1).flatten(0, 1)
        coords = _augment(2.0 * coords - 1.0, self, 2)
        return (2 * math.pi * coords[:, :, None] / self.periods[None, None, :]).flatten(1, 2)

    def forward(self, *, H: int, W: int) -> RopeTables:
        return RopeTables(self.angles(H=H, W=W))

    def _init_weights(self) -> None:
        self.periods.data = _geometric_periods(
            self.D_head // 4, self.D_head // 2, self.base, self.min_period, self.max_period, self.dtype,
            self.periods.device,
        )


class RopePositionEmbedding3D(_RopeBase):
    """3D vanilla: D_rope = (D_head // 6) * 6 channels on three axes; the remainder is unrotated."""

    periods: torch.Tensor

    def __init__(
        self,
        embed_dim: int,
        *,
        num_heads: int,
        base: float | None = 100.0,
        min_period: float | None = None,
        max_period: float | None = None,
        normalize_coords: Literal["min", "max", "separate"] = "separate",
        shift_coords: float | None = None,
        jitter_coords: float | None = None,
        rescale_coords: float | None = None,
        dtype: torch.dtype | None = None,
        device: torch.device | None = None,
    ) -> None:
        super().__init__()
        self._common_init(embed_dim, num_heads, base, min_period, max_period, normalize_coords, shift_coords,
                          jitter_coords, rescale_coords, dtype)
        if self.D_head % 2 != 0:
            raise ValueError(
                f"embed_dim {embed_dim} / num_heads {num_heads} gives an odd head dimension {self.D_head}; "
                "rotary embedding rotates channel pairs, so it must be even."
            )
        self.D_rope = (self.D_head // 6) * 6
        self.register_buffer("periods", torch.empty(self.D_rope // 6, device=device, dtype=dtype), persistent=True)
        self._init_weights()

    def angles(self, *, D: int, H: int, W: int) -> torch.Tensor:
        cd, ch, cw = _axis_coords((D, H, W), self.normalize_coords, self.dtype, self.periods.device)
        coords = torch.stack(torch.meshgrid(cd, ch, cw, indexing="ij"), dim=-1).flatten(0, 2)
        coords = _augment(2.0 * coords - 1.0, self, 3)
        angles = (2 * math.pi * coords[:, :, None] / self.periods[None, None, :]).flatten(1, 2)
        if self.D_rope < self.D_head:
            angles = F.pad(angles, (0, (self.D_head - self.D_rope) // 2))
        return angles

    def forward(self, *, D: int, H: int, W: int) -> RopeTables:
        return RopeTables(self.angles(D=D, H=H, W=W))

    def _init_weights(self) -> None:
        self.periods.data = _geometric_periods(
            self.D_rope // 6, self.D_rope // 3, self.base, self.min_period, self.max_period, self.dtype,
            self.periods.device,
        )


class RopePositionEmbedding3DSuperposition(_RopeBase):
    """The 2D layout on (H, W) plus `depth_scale` * a depth angle on every channel pair.

    `depth_scale` starts at zero, so a 2D checkpoint's rotation is reproduced exactly at init and
    the model learns how much depth to mix in.
    """

    periods: torch.Tensor
    depth_periods: torch.Tensor

    def __init__(
        self,
        embed_dim: int,
        *,
        num_heads: int,
        base: float | None = 100.0,
        depth_base: float | None = 10000.0,
        min_period: float | None = None,
        max_period: float | None = None,
        normalize_coords: Literal["min", "max", "separate"] = "separate",
        shift_coords: float | None = None,
        jitter_coords: float | None = None,
        rescale_coords: float | None = None,
        dtype: torch.dtype | None = None,
        device: torch.device | None = None,
    ) -> None:
        super().__init__()
        assert embed_dim % (4 * num_heads) == 0
        self._common_init(embed_dim, num_heads, base, min_period, max_period, normalize_coords, shift_coords,
                          jitter_coords, rescale_coords, dtype)
        self.depth_base = depth_base if depth_base is not None else base
        self.register_buffer("periods", torch.empty(self.D_head // 4, device=device, dtype=dtype), persistent=True)
        self.register_buffer("depth_periods", torch.empty(self.D_head // 4, device=device, dtype=dtype), persistent=True)
        self.depth_scale = nn.Parameter(torch.zeros(1, device=device, dtype=dtype))
        self._init_weights()

    def angles(self, *, D: int, H: int, W: int) -> torch.Tensor:
        dd = {"dtype": self.dtype, "device": self.periods.device}
        cd, ch, cw = _axis_coords((D, H, W), self.normalize_coords, self.dtype, self.periods.device)
        gd, gh, gw = torch.meshgrid(cd, ch, cw, indexing="ij")
        spatial = 2.0 * torch.stack([gh, gw], dim=-1).flatten(0, 2) - 1.0
        depth = 2.0 * gd.flatten(0, 2) - 1.0
        if self.training and self.shift_coords is not None:
            spatial = spatial + torch.empty(2, **dd).uniform_(-self.shift_coords, self.shift_coords)[None]
            depth = depth + torch.empty(1, **dd).uniform_(-self.shift_coords, self.shift_coords)
        if self.training and self.jitter_coords is not None:
            jmax = math.log(self.jitter_coords)
            spatial = spatial * torch.empty(2, **dd).uniform_(-jmax, jmax).exp()[None]
            depth = depth * torch.empty(1, **dd).uniform_(-jmax, jmax).exp()
        if self.training and self.rescale_coords is not None:
            rmax = math.log(self.rescale_coords)
            r = torch.empty(1, **dd).uniform_(-rmax, rmax).exp()
            spatial = spatial * r
            depth = depth * r
        a_sp = (2 * math.pi * spatial[:, :, None] / self.periods[None, None, :]).flatten(1, 2)
        a_d = (2 * math.pi * depth[:, None] / self.depth_periods[None, :]).repeat(1, 2)
        return a_sp + self.depth_scale * a_d

    def forward(self, *, D: int, H: int, W: int) -> RopeTables:
        return RopeTables(self.angles(D=D, H=H, W=W))

    def _init_weights(self) -> None:
        dev = self.periods.device
        self.periods.data = _geometric_periods(
            self.D_head // 4, self.D_head // 2, self.base, self.min_period, self.max_period, self.dtype, dev
        )
        if self.base is not None:
            self.depth_periods.data = _geometric_periods(
                self.D_head // 4, self.D_head // 2, self.depth_base, None, None, self.dtype, dev
            )
        else:
            self.depth_periods.data = self.periods.data.clone()
