"""Device-side input normalisation.

Volumes travel host -> device as uint8 (a quarter of the bytes of fp32) and are z-scored per
volume on the GPU: `zscore_u8` computes each volume's mean and unbiased standard deviation from
exact integer moments, then writes (x - mean) / max(std, 1e-6) in the compute dtype, in two
native kernels (`csrc/data_ops.cu`). The fallback for CPU tensors is the same formula in torch.
"""

from __future__ import annotations

import torch

from ._native import native, use_native


def zscore_u8_reference(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    v = x.double()
    dims = tuple(range(1, v.dim()))
    mean = v.mean(dim=dims, keepdim=True)
    std = v.std(dim=dims, keepdim=True).clamp_min(1e-6)
    return ((v - mean) / std).to(dtype)


def zscore_u8(x: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Per-volume z-score of a uint8 batch `(B, ...)` (statistics over all but the first axis)."""
    if x.dtype != torch.uint8:
        raise TypeError(f"zscore_u8 expects uint8 volumes, got {x.dtype}")
    if dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"zscore_u8 writes bf16 or fp32, not {dtype}")
    per_vol = x[0].numel() if x.shape[0] else 0
    if use_native(x) and x.is_contiguous() and (per_vol % 16 == 0 or x.shape[0] == 1):
        out = torch.empty(x.shape, device=x.device, dtype=dtype)
        native().zscore_u8(x, out)
        return out
    return zscore_u8_reference(x, dtype)
