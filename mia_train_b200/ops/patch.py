"""Volume <-> patch-token layout ops.

`patchify(volumes, patch, index)` turns (B, C, D, H, W) into (B, K, C*pd*ph*pw) rows in the order a
`Conv3d(kernel=stride=patch)` weight flattens to (channel, then the three patch axes), for the
patch indices `index` (B, K) in row-major grid order, or for every patch when `index` is None. On
CUDA one native kernel gathers and converts to the compute dtype in a single pass, which is what
lets masked autoencoding embed only its visible patches: a kernel==stride convolution is
independent per patch, so embedding a subset equals embedding everything and gathering.
"""

from __future__ import annotations

import torch

from ._native import native, use_native


def patchify_reference(volumes: torch.Tensor, patch: tuple[int, int, int]) -> torch.Tensor:
    b, c, d, h, w = volumes.shape
    pd, ph, pw = patch
    gd, gh, gw = d // pd, h // ph, w // pw
    x = volumes.reshape(b, c, gd, pd, gh, ph, gw, pw).permute(0, 2, 4, 6, 1, 3, 5, 7)
    return x.reshape(b, gd * gh * gw, c * pd * ph * pw)


def patchify(
    volumes: torch.Tensor,
    patch: tuple[int, int, int],
    index: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    out_dtype = out_dtype or volumes.dtype
    b, c, d, h, w = volumes.shape
    pd, ph, pw = patch
    if use_native(volumes) and volumes.dtype in (torch.float32, torch.bfloat16):
        grid = (d // pd, h // ph, w // pw)
        n = grid[0] * grid[1] * grid[2]
        if index is None:
            index = torch.arange(n, device=volumes.device, dtype=torch.int64).expand(b, n)
        k = index.shape[1]
        out = torch.empty((b, k, c * pd * ph * pw), device=volumes.device, dtype=out_dtype)
        native().patch_gather(volumes.contiguous(), index.to(torch.int64).contiguous(), out, pd, ph, pw)
        return out
    rows = patchify_reference(volumes, patch)
    if index is not None:
        rows = torch.gather(rows, 1, index.unsqueeze(-1).expand(-1, -1, rows.shape[-1]))
    return rows.to(out_dtype)
