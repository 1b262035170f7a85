"""Tensor parallelism for transformer blocks: head-sharded attention, column/row-sharded MLPs.

The reference drives TP through `parallelize_module(model, mesh["tp"], model.tensor_parallel_plan())`
(`src/distributed/parallelize.py:16-26`) but ships no plan (`src/models/base.py:126-128`). Here a
model's `tensor_parallel_plan()` returns a `BlockTensorParallelPlan`, applied in place:

* `attn.qkv` is column-parallel and **head-aligned**: rank r keeps the rows of its heads of q, of k
  and of v, so its local output reshapes to `(3, heads / tp, head_dim)` (a plain Shard(0) of the
  fused weight would mix q, k and v rows). The key-masked bias and its mask are sliced the same way.
* `attn.proj`, `mlp.fc2` / `mlp.2` / `mlp.w3` are row-parallel (columns of the local heads / hidden
  units); their bias is kept whole and added once, after the reduction.
* `mlp.fc1` / `mlp.0` / `mlp.w1` / `mlp.w2` are column-parallel.
* Norms, LayerScale, rotary frequencies and everything outside the blocks stay replicated.

Collectives (Megatron form): a column-parallel layer's input passes `copy_to_tp` (identity forward,
gradient all-reduce backward), a row-parallel layer's output passes `reduce_from_tp` (all-reduce
forward, identity backward), and the rotary angles, which feed only the local heads, pass
`copy_to_tp` too. Every replicated parameter therefore receives the full gradient on every rank
and needs no extra synchronisation. The local GEMMs are the native tcgen05 GEMMs.

Checkpoints keep the unsharded layout: the state-dict hook all-gathers each sharded tensor over the
TP group (undoing the head grouping of qkv) and the load hook slices a full tensor back, so a TP run
saves and loads the same files as a single-GPU run.
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x: torch.Tensor, group: Any) -> torch.Tensor:
    return _CopyToTP.apply(x, group)


def reduce_from_tp(x: torch.Tensor, group: Any) -> torch.Tensor:
    return _ReduceFromTP.apply(x, group)


@dataclass
class BlockTensorParallelPlan:
    """Which submodules of each block are column / row / qkv-parallel (attribute paths)."""

    blocks: list[nn.Module]
    qkv: tuple[str, ...] = ("attn.qkv",)
    column: tuple[str, ...] = ("mlp.fc1", "mlp.0", "mlp.w1", "mlp.w2")
    row: tuple[str, ...] = ("attn.proj", "mlp.fc2", "mlp.2", "mlp.w3")
    attention: tuple[str, ...] = ("attn",)
    prefix: str = "blocks"
    extra: dict[str, Any] = field(default_factory=dict)


def vit_block_plan(blocks: Iterable[nn.Module], prefix: str = "blocks") -> BlockTensorParallelPlan:
    return BlockTensorParallelPlan(blocks=list(blocks), prefix=prefix)


def _get(module: nn.Module, path: str) -> nn.Module | None:
    cur: Any = module
    for part in path.split("."):
        if isinstance(cur, nn.Sequential) and part.isdigit():
            idx = int(part)
            if idx >= len(cur):
                return None
            cur = cur[idx]
        elif hasattr(cur, part):
            cur = getattr(cur, part)
        else:
            return None
    return cur if isinstance(cur, nn.Module) else None


def _qkv_rows(out3: int, rank: int, world: int) -> torch.Tensor:
    """Row indices of rank `rank`'s q, k and v blocks in a fused (3C, .) qkv weight."""
    c = out3 // 3
    per = c // world
    idx = [torch.arange(part * c + rank * per, part * c + (rank + 1) * per) for part in range(3)]
    return torch.cat(idx)


def _chunk(n: int, rank: int, world: int) -> slice:
    per = n // world
    return slice(rank * per, (rank + 1) * per)


def _replace(module: nn.Module, name: str, value: torch.Tensor) -> None:
    old = getattr(module, name)
    if isinstance(old, nn.Parameter):
        setattr(module, name, nn.Parameter(value.contiguous(), requires_grad=old.requires_grad))
    else:
        module.register_buffer(name, value.contiguous(), persistent=name in module.state_dict())


@torch.no_grad()
def _shard_linear(lin: nn.Linear, mode: str, rank: int, world: int, group: Any) -> None:
    w = lin.weight
    if mode == "qkv":
        if w.shape[0] % (3 * world):
            raise ValueError(f"qkv rows {w.shape[0]} are not divisible by 3 * tp = {3 * world}")
        rows = _qkv_rows(w.shape[0], rank, world).to(w.device)
        _replace(lin, "weight", w.index_select(0, rows))
        if lin.bias is not None:
            _replace(lin, "bias", lin.bias.index_select(0, rows))
        if hasattr(lin, "bias_mask") and isinstance(lin.bias_mask, torch.Tensor):
            _replace(lin, "bias_mask", lin.bias_mask.index_select(0, rows))
    elif mode == "column":
        if w.shape[0] % world:
            raise ValueError(f"{w.shape[0]} output features are not divisible by tp = {world}")
        s = _chunk(w.shape[0], rank, world)
        _replace(lin, "weight", w[s])
        if lin.bias is not None:
            _replace(lin, "bias", lin.bias[s])
    elif mode == "row":
        if w.shape[1] % world:
            raise ValueError(f"{w.shape[1]} input features are not divisible by tp = {world}")
        _replace(lin, "weight", w[:, _chunk(w.shape[1], rank, world)])
    else:  # pragma: no cover - internal
        raise ValueError(mode)
    lin._tp_mode = mode  # type: ignore[attr-defined]
    lin._tp_group = group  # type: ignore[attr-defined]
    lin._tp_world = world  # type: ignore[attr-defined]
    lin._tp_rank = rank  # type: ignore[attr-defined]


def tp_linear(
    module: nn.Linear,
    x: torch.Tensor,
    activation: str | None = None,
    residual: torch.Tensor | None = None,
    gamma: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """The sharded layer's part of `residual + gamma * act(module(x))`, collectives included."""
    from ..ops.linear import linear

    mode = module._tp_mode  # type: ignore[attr-defined]
    group = module._tp_group  # type: ignore[attr-defined]
    b = module.bias if bias is None else bias
    if mode in ("qkv", "column"):
        if residual is not None or gamma is not None:
            raise ValueError("a column-parallel layer cannot take a residual or LayerScale")
        return linear(copy_to_tp(x, group), module.weight, b, activation=activation)
    if activation is not None:
        raise ValueError("a row-parallel layer cannot apply an activation before its reduction")
    y = reduce_from_tp(linear(x, module.weight, None), group)
    if b is not None:
        y = y + b.to(y.dtype)
    if gamma is not None:
        y = y * gamma.to(y.dtype)
    return y if residual is None else residual + y


def is_tensor_parallel(module: nn.Module) -> bool:
    return hasattr(module, "_tp_mode")


def _state_hooks(block: nn.Module, prefix_paths: dict[str, str], group: Any, rank: int, world: int) -> None:
    """Save whole tensors (all-gathered over TP) and slice whole tensors on load."""
    modes = dict(prefix_paths)

    def full(local: torch.Tensor, mode: str, name: str) -> torch.Tensor:
        t = local.full_tensor() if hasattr(local, "full_tensor") else local
        t = t.detach().contiguous()
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t, group=group)
        if mode == "qkv":  # undo the head grouping: (rank, part, rows) -> (part, rank, rows)
            per = t.shape[0] // 3
            return torch.cat([parts[r][p * per:(p + 1) * per] for p in range(3) for r in range(world)])
        if mode == "column" or name != "weight":
            return torch.cat(parts, dim=0)
        return torch.cat(parts, dim=1)

    def save_hook(module, state_dict, prefix, local_metadata):
        for path, mode in modes.items():
            for name in ("weight", "bias", "bias_mask"):
                key = f"{prefix}{path}.{name}"
                if key not in state_dict:
                    continue
                if mode == "row" and name != "weight":
                    continue  # replicated
                state_dict[key] = full(state_dict[key], mode, name)
        return state_dict

    def load_hook(module, state_dict, prefix, local_metadata, strict, missing, unexpected, errors):
        for path, mode in modes.items():
            lin = _get(module, path)
            for name in ("weight", "bias", "bias_mask"):
                key = f"{prefix}{path}.{name}"
                if key not in state_dict or lin is None or getattr(lin, name, None) is None:
                    continue
                src = state_dict[key]
                if src.shape == getattr(lin, name).shape:
                    continue  # already local
                if mode == "qkv":
                    state_dict[key] = src.index_select(0, _qkv_rows(src.shape[0], rank, world).to(src.device))
                elif mode == "column":
                    state_dict[key] = src[_chunk(src.shape[0], rank, world)]
                elif name == "weight":
                    state_dict[key] = src[:, _chunk(src.shape[1], rank, world)]

    block._register_state_dict_hook(save_hook)
    block._register_load_state_dict_pre_hook(load_hook, with_module=True)


def apply_tensor_parallel(plan: BlockTensorParallelPlan, group: Any) -> int:
    """Shard every block of `plan` in place over `group`; returns the number of sharded layers."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    count = 0
    for block in plan.blocks:
        modes: dict[str, str] = {}
        for mode, paths in (("qkv", plan.qkv), ("column", plan.column), ("row", plan.row)):
            for path in paths:
                lin = _get(block, path)
                if isinstance(lin, nn.Linear):
                    if is_tensor_parallel(lin):
                        raise ValueError(f"{path} is already tensor-parallel")
                    _shard_linear(lin, mode, rank, world, group)
                    modes[path] = mode
                    count += 1
        for path in plan.attention:
            attn = _get(block, path)
            if attn is not None:
                localize_attention(attn, world, group)
        _state_hooks(block, modes, group, rank, world)
    return count


def localize_attention(attn: nn.Module, world: int, group: Any) -> None:
    heads = int(attn.num_heads)
    if heads % world:
        raise ValueError(f"{heads} attention heads are not divisible by tp = {world}")
    attn.num_heads = heads // world
    attn._tp_group = group  # type: ignore[attr-defined]


def localize_heads(blocks: Iterable[nn.Module], world: int) -> None:
    """Kept for plans applied through `parallelize_module`: heads per rank after sharding."""
    for block in blocks:
        attn = getattr(block, "attn", None)
        if attn is not None and not hasattr(attn, "_tp_group"):
            attn.num_heads = int(attn.num_heads) // world


def rope_to_tp(angles: torch.Tensor | None, module: nn.Module) -> torch.Tensor | None:
    """Angles feeding only this rank's heads: their gradient is summed over the TP group."""
    group = getattr(module, "_tp_group", None)
    if angles is None or group is None or not angles.requires_grad:
        return angles
    return copy_to_tp(angles, group)
