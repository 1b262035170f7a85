"""Dense heads: patch-grid features -> one prediction per voxel (reference `src/layers/common/dense_heads.py:46-286`).

Both heads take `forward(x, size)` with `x` shaped `(B, C, *grid)` and return `(B, out, *size)`,
and both change resolution inside the module, so an activation-checkpointed head stores only its
patch-grid input.

`VoxelHead` (an `nn.Sequential` of the layers that run at voxel resolution) upsamples with
separable linear interpolation written as one fp32 matrix product per axis. The `(target, extent)`
matrices are built here from the half-pixel convention of `F.interpolate(mode="linear",
align_corners=False)`: source coordinate `(o + 0.5) * extent / target - 0.5`, clamped below at 0,
the two nearest cells weighted linearly and the upper index clamped at `extent - 1`. A matmul's
backward is a matmul, so there is no scatter-add contention in the gradient; the matrices are a
per-(extent, target, device) cache, not state.

`SubPixelHead` projects (1x1 conv), expands every token into its own `readout x patch` block with
a transposed convolution whose kernel equals its stride, refines with `refine_depth` 3-wide
convolutions + GELU and maps to the outputs with a 1x1 conv. The expansion is evaluated as one
GEMM over tokens, `(B*N, hidden) @ (hidden, readout * prod(patch))`, on the native tcgen05 GEMM
when the activations are bf16 on CUDA, followed by a fold that interleaves each grid axis with its
in-block offset. Parameters keep the transposed-convolution layout and names (`expand.weight`
`(hidden, readout, *patch)`, `expand.bias`), so checkpoints are interchangeable.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from ...ops.linear import compute_dtype, linear

CONV: dict[int, Any] = {2: nn.Conv2d, 3: nn.Conv3d}
CONV_TRANSPOSE: dict[int, Any] = {2: nn.ConvTranspose2d, 3: nn.ConvTranspose3d}
INTERPOLATION = {2: "bilinear", 3: "trilinear"}


def linear_resample_matrix(extent: int, target: int, device: torch.device | None = None) -> torch.Tensor:
    """(target, extent) fp32 matrix of 1-D linear interpolation with half-pixel centres."""
    out = torch.arange(target, dtype=torch.float64)
    src = ((out + 0.5) * (extent / target) - 0.5).clamp_min(0.0)
    lo = src.floor().long().clamp_max(extent - 1)
    frac = src - lo.double()
    hi = (lo + 1).clamp_max(extent - 1)
    m = torch.zeros(target, extent, dtype=torch.float64)
    rows = torch.arange(target)
    m.index_put_((rows, lo), 1.0 - frac, accumulate=True)
    m.index_put_((rows, hi), frac, accumulate=True)
    return m.to(device=device, dtype=torch.float32)


class VoxelHead(nn.Sequential):
    def __init__(self, *layers: nn.Module, mode: str = "trilinear") -> None:
        super().__init__(*layers)
        self.mode = mode
        self._matrices: dict[tuple[int, int, torch.device], torch.Tensor] = {}

    def _matrix(self, extent: int, target: int, device: torch.device) -> torch.Tensor:
        key = (extent, target, device)
        m = self._matrices.get(key)
        if m is None:
            m = linear_resample_matrix(extent, target, device)
            self._matrices[key] = m
        return m

    def upsample(self, x: torch.Tensor, size: tuple[int, ...]) -> torch.Tensor:
        """(B, C, *grid) -> (B, C, *size), fp32, one matmul per axis (last axis first)."""
        with torch.autocast(x.device.type, enabled=False):
            x = x.float()
            for axis in reversed(range(len(size))):
                m = self._matrix(x.shape[-1], size[axis], x.device)
                # resample the trailing axis and rotate it to the front of the spatial block
                x = torch.matmul(x, m.t()).movedim(-1, 2)
        return x

    def forward(self, x: torch.Tensor, size: tuple[int, ...]) -> torch.Tensor:  # type: ignore[override]
        x = self.upsample(x, tuple(size))
        if not torch.is_autocast_enabled(x.device.type):
            # the upsampling ran in fp32; the layers may hold lower-precision parameters (FSDP's
            # compute dtype) and there is no autocast to cast the input for them
            w = next((p for p in self.parameters() if p.is_floating_point()), None)
            if w is not None and w.dtype != x.dtype:
                x = x.to(w.dtype)
        for layer in self:
            x = layer(x)
        return x


class SubPixelHead(nn.Module):
    def __init__(
        self,
        in_dim: int,
        patch_size: tuple[int, ...],
        out_channels: int,
        hidden: int = 256,
        readout: int = 16,
        refine_depth: int = 2,
        zero_init_output: bool = True,
    ) -> None:
        super().__init__()
        rank = len(patch_size)
        if rank not in CONV:
            raise ValueError(f"patch_size must have 2 or 3 entries, got {patch_size}")
        if refine_depth < 1:
            raise ValueError(
                f"refine_depth must be at least 1, got {refine_depth}: some convolution after the expansion "
                "has to mix values across neighbouring token blocks"
            )
        self.patch_size = tuple(int(p) for p in patch_size)
        conv, conv_t = CONV[rank], CONV_TRANSPOSE[rank]
        self.project = conv(in_dim, hidden, kernel_size=1)
        self.expand = conv_t(hidden, readout, kernel_size=self.patch_size, stride=self.patch_size)
        if tuple(self.expand.kernel_size) != tuple(self.expand.stride):
            raise ValueError("SubPixelHead needs kernel_size == stride: the expansion is a per-token GEMM")
        layers: list[nn.Module] = []
        for _ in range(refine_depth):
            layers += [conv(readout, readout, kernel_size=3, padding=1), nn.GELU()]
        self.refine = nn.Sequential(*layers)
        self.out = conv(readout, out_channels, kernel_size=1)
        if zero_init_output:
            nn.init.zeros_(self.out.weight)
        nn.init.zeros_(self.out.bias)

    def set_output_bias(self, bias: float) -> None:
        nn.init.constant_(self.out.bias, bias)

    def expand_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """`self.expand(x)` as a token GEMM plus fold: (B, hidden, *grid) -> (B, readout, *grid*patch)."""
        b, hidden, *grid = x.shape
        rank = len(grid)
        readout = self.expand.out_channels
        tokens = x.flatten(2).transpose(1, 2)  # (B, N, hidden)
        # weight (hidden, readout, *patch) -> (readout*prod(patch), hidden): a Linear weight
        w = self.expand.weight.reshape(hidden, -1).t()
        if x.is_cuda and compute_dtype(x) == torch.bfloat16:
            y = linear(tokens.to(torch.bfloat16).contiguous(), w.contiguous(), None)
        else:
            y = tokens @ w.t().to(tokens.dtype)
        y = y.reshape(b, *grid, readout, *self.patch_size)
        order = [0, rank + 1]
        for axis in range(rank):
            order += [1 + axis, rank + 2 + axis]
        y = y.permute(*order).reshape(b, readout, *[g * p for g, p in zip(grid, self.patch_size, strict=True)])
        if self.expand.bias is not None:
            y = y + self.expand.bias.to(y.dtype).reshape(readout, *(1,) * rank)
        return y

    def forward(self, x: torch.Tensor, size: tuple[int, ...]) -> torch.Tensor:
        covered = tuple(g * p for g, p in zip(x.shape[2:], self.patch_size, strict=True))
        if tuple(size) != covered:
            raise ValueError(
                f"a patch grid of {tuple(x.shape[2:])} at patch size {self.patch_size} covers {covered}, but the "
                f"crop is {tuple(size)}; the sub-pixel head needs a crop divisible by the patch size"
            )
        x = self.project(x)
        x = self.expand_tokens(x)
        x = self.refine(x)
        return self.out(x)
