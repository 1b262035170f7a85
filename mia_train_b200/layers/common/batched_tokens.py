"""Concatenate a list of crops' tokens to one (sum N, C) matrix and split it back (reference
`src/layers/common/batched_tokens.py:19-44`): list-batched crops share one GEMM per projection."""

from __future__ import annotations

import torch


def cat_keep_shapes(x_list: list[torch.Tensor]) -> tuple[torch.Tensor, list[torch.Size], list[int]]:
    shapes = [x.shape for x in x_list]
    counts = [x.numel() // x.shape[-1] for x in x_list]
    flat = torch.cat([x.reshape(-1, x.shape[-1]) for x in x_list], dim=0)
    return flat, shapes, counts


def uncat_with_shapes(flat: torch.Tensor, shapes: list[torch.Size], counts: list[int]) -> list[torch.Tensor]:
    parts = torch.split(flat, counts, dim=0)
    return [p.reshape(*s[:-1], flat.shape[-1]) for p, s in zip(parts, shapes, strict=True)]
