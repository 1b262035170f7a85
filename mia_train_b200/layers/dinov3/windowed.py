"""Windowed 3D attention for DINOv3 blocks (new; the reference's attention is always global).

A windowed block partitions the patch grid (D, H, W) into non-overlapping `w^3` windows. Patch
tokens attend to the tokens of their own window plus the prefix tokens (class + registers), which
every window can see; prefix tokens attend globally. Everything outside attention (norms,
projections, MLP, LayerScale, residuals) is per token and identical to the global block. RoPE uses
the same per-token angles as the global block, so position encoding is unchanged.

Cost per block: `N (w^3 + P)` key interactions instead of `N^2` -- for a 32^3 grid with 8^3 windows,
64x fewer.
"""

from __future__ import annotations

import functools

import torch
import torch.nn.functional as F

from ...ops.attention import attention, rope_attention
from ...parallel.tensor_parallel import rope_to_tp
from .block import SelfAttentionBlock
from .rope import RopeTables


def window_partition(x: torch.Tensor, grid: tuple[int, int, int], w: int) -> torch.Tensor:
    """(B, D*H*W, C) row-major grid tokens -> (B * nw, w^3, C) windows."""
    b, _, c = x.shape
    d, h, ww = grid
    x = x.reshape(b, d // w, w, h // w, w, ww // w, w, c).permute(0, 1, 3, 5, 2, 4, 6, 7)
    return x.reshape(-1, w * w * w, c)


def window_merge(x: torch.Tensor, b: int, grid: tuple[int, int, int], w: int) -> torch.Tensor:
    """Inverse of `window_partition`."""
    d, h, ww = grid
    c = x.shape[-1]
    x = x.reshape(b, d // w, h // w, ww // w, w, w, w, c).permute(0, 1, 4, 2, 5, 3, 6, 7)
    return x.reshape(b, d * h * ww, c)


def windowed_attention(
    attn,
    qkv: torch.Tensor,
    grid: tuple[int, int, int],
    rope: RopeTables | None,
    n_prefix: int,
    w: int,
) -> torch.Tensor:
    """(B, P + N, 3 C) projections -> (B, P + N, C): patch queries attend within their window plus the
    prefix tokens, prefix queries attend to every token. C is this rank's share of the width under
    tensor parallelism."""
    if any(g % w for g in grid):
        raise ValueError(f"patch grid {grid} is not divisible by window_size {w}")
    b, n_tok, _ = qkv.shape
    heads, hd = attn.num_heads, attn.head_dim
    c = heads * hd
    pre, pat = qkv[:, :n_prefix], qkv[:, n_prefix:]
    nwin = (grid[0] // w) * (grid[1] // w) * (grid[2] // w)
    win = window_partition(pat, grid, w)  # (B*nw, w^3, 3C)
    # prefix rows for every window: a broadcast (its backward is a sum over windows; an index-based
    # repeat would back-propagate through a sorted scatter with 64-fold duplicate indices)
    pre_rep = pre.unsqueeze(1).expand(b, nwin, n_prefix, pre.shape[-1]).reshape(b * nwin, n_prefix, pre.shape[-1])
    pre_rep = pre_rep.contiguous()  # with B = 1 the reshape is a stride-0 view, which takes cat's slow path
    packed = torch.cat([pre_rep, win], dim=1).reshape(b * nwin, n_prefix + w**3, 3, heads, hd)
    angles_win = pairs = None
    if rope is not None:
        ang = rope_to_tp(rope.angles.float(), attn)  # (N, D/2)
        ang_w = window_partition(ang.unsqueeze(0), grid, w)  # (nw, w^3, D/2)
        ang_w = F.pad(ang_w, (0, 0, n_prefix, 0))
        angles_win = ang_w.repeat(b, 1, 1)
        pairs = attn._pairs_on(qkv.device)
    out_win = rope_attention(packed, angles_win, pairs, attn.scale)[:, n_prefix:]  # (B*nw, w^3, H, hd)
    out_pat = window_merge(out_win.reshape(b * nwin, w**3, c), b, grid, w)
    # prefix queries attend to every token (keys of patches rotated by their angles)
    q_pre = pre[..., :c].reshape(b, n_prefix, heads, hd)
    k_all = qkv[..., c : 2 * c].reshape(b, n_tok, heads, hd)
    v_all = qkv[..., 2 * c :].reshape(b, n_tok, heads, hd)
    if rope is not None:
        full = F.pad(rope_to_tp(rope.angles.float(), attn), (0, 0, n_prefix, 0)).unsqueeze(0)
        k_all = rotate_half(k_all, full)
    out_pre = attention(q_pre.contiguous(), k_all.contiguous(), v_all.contiguous(), attn.scale).reshape(b, n_prefix, c)
    return torch.cat([out_pre, out_pat.to(out_pre.dtype)], dim=1)


def rotate_half(x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """RoPE with channel pairs (i, i + D / 2) on (B, N, H, D) by (1 or B, N, D / 2) angles, written with
    slices only, so its backward is elementwise (an index-based rotation back-propagates through a
    sorted scatter)."""
    half = x.shape[-1] // 2
    cos = angles.cos().unsqueeze(-2)
    sin = angles.sin().unsqueeze(-2)
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def windowed_core(grid: tuple[int, int, int], rope: RopeTables | None, n_prefix: int, w: int):
    """The attention core of a windowed block, for `SelfAttentionBlock.forward(..., attention=...)`."""
    return functools.partial(_windowed_core, grid=grid, rope=rope, n_prefix=n_prefix, w=w)


def _windowed_core(attn, qkv, *, grid, rope, n_prefix, w):
    return windowed_attention(attn, qkv, grid, rope, n_prefix, w)


def windowed_block_forward(
    blk: SelfAttentionBlock,
    x: torch.Tensor,
    grid: tuple[int, int, int],
    rope: RopeTables | None,
    n_prefix: int,
    w: int,
) -> torch.Tensor:
    """One block (or its activation-checkpoint wrapper) with windowed attention."""
    return blk(x, rope, attention=windowed_core(grid, rope, n_prefix, w))
