"""Sequence-parallel tensor parallelism for transformer blocks (Megatron-SP layout).

Inside a block the residual stream stays sharded by token: rank r of the TP group holds rows
[r S, (r + 1) S) of the (B * T_pad, C) token matrix (`T_pad` = tokens rounded up to a multiple of
128 x the TP size, so every rank holds whole 128-row blocks; the padding rows never reach
attention or the loss). LayerNorms, LayerScale and the
residual adds run on the shard. The block's four GEMMs are

    qkv  = gather(LN1(x)) . Wqkv_r^T           column-parallel, all-gather -> GEMM
    x    = x + ls1 * scatter(attn . Wproj_r^T)  row-parallel,    GEMM -> reduce-scatter
    u    = gelu(gather(LN2(x)) . W1_r^T)        column-parallel, all-gather -> GEMM
    x    = x + ls2 * scatter(u . W2_r^T)        row-parallel,    GEMM -> reduce-scatter

and backward mirrors them (dX of a column-parallel layer is a GEMM -> reduce-scatter, dX of a
row-parallel layer an all-gather -> GEMM whose gathered operand also feeds the weight gradient).
With `TpComm("fused")` each of these is one native kernel moving data over NVLink peer memory
from inside the GEMM (`ops/tp.py`, `csrc/tp_gemm.cu`); with `TpComm("collective")` they are
NCCL (or Gloo) collectives around the GEMMs.

Parameter gradients: the sharded weights and the biases of the column-parallel layers are
complete on their rank; the biases of the row-parallel layers are summed over the gathered output
gradient, so they are complete too. LayerNorm weights / biases and LayerScale gammas see only this
rank's tokens: their modules are marked `_sp_partial_group` and `sync_partial_grads` sums them
over the TP group (one all-reduce) after backward. Attention runs on all tokens of the local heads, as in the
non-sequence-parallel layout (`parallel/tensor_parallel.py`).
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from ..ops._params import compute_weight, grad_sink
from ..ops.linear import ACT_DGELU, ACT_GELU, column_sum, compute_dtype, gemm
from ..ops.tp import TpComm, ag_gemm, gemm_rs


def _weight_grad(dout, inp, sink, wshape, wdtype):
    if sink is not None:
        gemm(dout, inp, a_kmajor=False, b_kmajor=False, out=sink.view(wshape), accumulate=True)
        return None
    return gemm(dout, inp, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32).to(wdtype).view(wshape)


def _bias_grad(dout, sink, present, dtype):
    if not present:
        return None
    if sink is not None:
        column_sum(dout, out=sink, accumulate=True)
        return None
    return column_sum(dout).to(dtype)


def _f32(t: torch.Tensor | None) -> torch.Tensor | None:
    return t.float().contiguous() if t is not None else None


class _ColumnParallel(torch.autograd.Function):
    """y = gather(x_r) . W^T + b over the TP group (qkv)."""

    @staticmethod
    def forward(ctx, x, weight, bias, comm, cdtype):  # type: ignore[override]
        xs = x.to(cdtype).contiguous()
        w = compute_weight(weight, cdtype).contiguous()
        y, full, _ = ag_gemm(comm, xs, w, bias=_f32(bias))
        ctx.save_for_backward(full, w)
        ctx.comm = comm
        ctx.meta = (bias is not None, weight.dtype, bias.dtype if bias is not None else None, weight.shape)
        ctx.sinks = (grad_sink(weight), grad_sink(bias))
        return y

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        full, w = ctx.saved_tensors
        has_b, wdtype, bdtype, wshape = ctx.meta
        sw, sb = ctx.sinks
        dy = dy.to(full.dtype).contiguous()
        dx, _ = gemm_rs(ctx.comm, dy, w, b_kmajor=False)
        dw = _weight_grad(dy, full, sw, wshape, wdtype) if ctx.needs_input_grad[1] else None
        db = _bias_grad(dy, sb, has_b and ctx.needs_input_grad[2], bdtype)
        return dx, dw, db, None, None


class _RowParallel(torch.autograd.Function):
    """out_r = residual_r + gamma * (scatter(x . W^T) + b) over the TP group (proj)."""

    @staticmethod
    def forward(ctx, x, weight, bias, gamma, residual, comm, cdtype):  # type: ignore[override]
        xs = x.to(cdtype).contiguous()
        w = compute_weight(weight, cdtype).contiguous()
        res = residual.to(cdtype).contiguous() if residual is not None else None
        g = _f32(gamma)
        out, pre = gemm_rs(comm, xs, w, bias=_f32(bias), gamma=g, residual=res, want_pre=gamma is not None)
        ctx.save_for_backward(xs, w, pre, g)
        ctx.comm = comm
        ctx.meta = (bias is not None, residual is not None, gamma is not None, weight.dtype,
                    bias.dtype if bias is not None else None, weight.shape)
        ctx.sinks = (grad_sink(weight), grad_sink(bias))
        return out

    @staticmethod
    def backward(ctx, dout):  # type: ignore[override]
        xs, w, pre, g = ctx.saved_tensors
        has_b, has_res, has_g, wdtype, bdtype, wshape = ctx.meta
        sw, sb = ctx.sinks
        dout = dout.to(xs.dtype).contiguous()
        dgamma = None
        dz = dout
        if has_g:
            dgamma = (dout.float() * pre.float()).sum(0)
            dz = (dout.float() * g).to(xs.dtype)
        dx, dz_full, _ = ag_gemm(ctx.comm, dz, w, b_kmajor=False)
        dw = _weight_grad(dz_full, xs, sw, wshape, wdtype) if ctx.needs_input_grad[1] else None
        db = _bias_grad(dz_full, sb, has_b and ctx.needs_input_grad[2], bdtype)
        return dx, dw, db, dgamma, (dout if has_res else None), None, None


class _Mlp(torch.autograd.Function):
    """out_r = residual_r + gamma * (scatter(gelu(gather(x_r) . W1^T + b1) . W2^T) + b2)."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, gamma, residual, comm, cdtype):  # type: ignore[override]
        xs = x.to(cdtype).contiguous()
        w1c = compute_weight(w1, cdtype).contiguous()
        w2c = compute_weight(w2, cdtype).contiguous()
        u, full, pre = ag_gemm(comm, xs, w1c, bias=_f32(b1), act=ACT_GELU, want_pre=True)
        res = residual.to(cdtype).contiguous() if residual is not None else None
        g = _f32(gamma)
        out, pre2 = gemm_rs(comm, u, w2c, bias=_f32(b2), gamma=g, residual=res, want_pre=gamma is not None)
        ctx.save_for_backward(full, w1c, w2c, pre, u, pre2, g)
        ctx.comm = comm
        ctx.meta = (b1 is not None, b2 is not None, residual is not None, gamma is not None, w1.dtype, w2.dtype,
                    b1.dtype if b1 is not None else None, b2.dtype if b2 is not None else None, w1.shape, w2.shape)
        ctx.sinks = (grad_sink(w1), grad_sink(b1), grad_sink(w2), grad_sink(b2))
        return out

    @staticmethod
    def backward(ctx, dout):  # type: ignore[override]
        full, w1, w2, pre, u, pre2, g = ctx.saved_tensors
        has_b1, has_b2, has_res, has_g, w1dt, w2dt, b1dt, b2dt, w1s, w2s = ctx.meta
        sw1, sb1, sw2, sb2 = ctx.sinks
        dout = dout.to(full.dtype).contiguous()
        dgamma = None
        dz = dout
        if has_g:
            dgamma = (dout.float() * pre2.float()).sum(0)
            dz = (dout.float() * g).to(full.dtype)
        # dH = (gather(dz) . W2) * gelu'(pre); the gathered dz also feeds dW2 and db2.
        dh, dz_full, _ = ag_gemm(ctx.comm, dz, w2, b_kmajor=False, act=ACT_DGELU, aux=pre)
        dw2 = _weight_grad(dz_full, u, sw2, w2s, w2dt)
        db2 = _bias_grad(dz_full, sb2, has_b2, b2dt)
        dx, _ = gemm_rs(ctx.comm, dh, w1, b_kmajor=False)
        dw1 = _weight_grad(dh, full, sw1, w1s, w1dt)
        db1 = _bias_grad(dh, sb1, has_b1, b1dt)
        return dx, dw1, db1, dw2, db2, dgamma, (dout if has_res else None), None, None


class _SplitRows(torch.autograd.Function):
    """Replicated (M, C) -> this rank's (M / W, C) rows; backward all-gathers the row gradients."""

    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        ctx.group = group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        rows = x.shape[0] // world
        return x[rank * rows:(rank + 1) * rows].contiguous()

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        world = dist.get_world_size(ctx.group)
        if world == 1:
            return g, None
        parts = [torch.empty_like(g) for _ in range(world)]
        dist.all_gather(parts, g.contiguous(), group=ctx.group)
        return torch.cat(parts, dim=0), None


class _GatherRows(torch.autograd.Function):
    """This rank's rows -> replicated (M, C); the computation after it is replicated over the TP group,
    so every rank receives the same output gradient and keeps its own rows of it."""

    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        ctx.group = group
        world = dist.get_world_size(group)
        if world == 1:
            return x.clone()
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=0)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        world, rank = dist.get_world_size(ctx.group), dist.get_rank(ctx.group)
        rows = g.shape[0] // world
        return g[rank * rows:(rank + 1) * rows].contiguous(), None


class _GatherRowsSummed(torch.autograd.Function):
    """This rank's rows -> all rows, for computation after it that each TP rank runs on a different
    part of the batch: the ranks' output gradients differ, so backward sums them over the group and
    keeps this rank's rows (a reduce-scatter)."""

    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        ctx.group = group
        world = dist.get_world_size(group)
        if world == 1:
            return x.clone()
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=0)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        from ..ops.tp import _scatter_sum_rows

        return _scatter_sum_rows(g, ctx.group), None


@dataclass
class SequenceParallel:
    """What a model needs to run its blocks sequence-parallel over one TP group.

    `split_samples`: while True, the computation after the blocks runs on a different slice of the
    batch on every TP rank (see `sample_slice`), so the final gather sums the ranks' gradients
    instead of assuming they are equal.
    """

    comm: TpComm
    split_samples: bool = False

    @property
    def world(self) -> int:
        return self.comm.world

    @property
    def group(self) -> Any:
        return self.comm.group

    def padded_tokens(self, t: int) -> int:
        """Tokens rounded up so every rank holds whole 128-row blocks (the fused kernels' unit)."""
        unit = self.world * 128 if self.world > 1 else 1
        return -(-t // unit) * unit

    def split(self, x: torch.Tensor) -> tuple[torch.Tensor, int]:
        """(B, T, C) replicated -> (this rank's rows of B * T_pad, C), T."""
        b, t, c = x.shape
        tp = self.padded_tokens(t)
        if tp != t:
            x = torch.nn.functional.pad(x, (0, 0, 0, tp - t))
        return _SplitRows.apply(x.reshape(b * tp, c), self.group), t

    def sample_slice(self, batch: int) -> slice | None:
        """This rank's samples of a batch split over the TP group: rank r of W takes samples
        [r B // W, (r + 1) B // W). None for a group of one; a batch smaller than the group is an
        error, since some rank would get no sample."""
        if self.world == 1:
            return None
        if batch < self.world:
            raise ValueError(f"a batch of {batch} cannot be split over a tensor-parallel group of {self.world}")
        rank = dist.get_rank(self.group)
        return slice(rank * batch // self.world, (rank + 1) * batch // self.world)

    def gather(self, x_r: torch.Tensor, b: int, t: int) -> torch.Tensor:
        full = (_GatherRowsSummed if self.split_samples else _GatherRows).apply(x_r, self.group)
        tp = full.shape[0] // b
        return full.reshape(b, tp, -1)[:, :t]


def column_parallel(x, weight, bias, sp: SequenceParallel):
    return _ColumnParallel.apply(x, weight, bias, sp.comm, compute_dtype(x))


def row_parallel(x, weight, bias, gamma, residual, sp: SequenceParallel):
    return _RowParallel.apply(x, weight, bias, gamma, residual, sp.comm, compute_dtype(x))


def mlp_parallel(x, w1, b1, w2, b2, gamma, residual, sp: SequenceParallel):
    return _Mlp.apply(x, w1, b1, w2, b2, gamma, residual, sp.comm, compute_dtype(x))


def block_forward(
    blk: nn.Module,
    x_r: torch.Tensor,
    sp: SequenceParallel,
    attention: Callable[[torch.Tensor], torch.Tensor],
    b: int,
    t: int,
) -> torch.Tensor:
    """One pre-norm block on this rank's token rows; `attention` maps the (B, T, 3 C_local) projection
    of all tokens (local heads) to the (B, T, C_local) attention output."""
    from ..ops.norm import layer_norm_residual

    attn, mlp = blk.attn, blk.mlp
    ls1 = getattr(blk.ls1, "gamma", None)
    ls2 = getattr(blk.ls2, "gamma", None)
    h, res = layer_norm_residual(x_r, blk.norm1.weight, blk.norm1.bias, blk.norm1.eps)
    qkv_bias = attn.qkv.masked_bias() if hasattr(attn.qkv, "masked_bias") else attn.qkv.bias
    qkv = column_parallel(h, attn.qkv.weight, qkv_bias, sp)  # (B * T_pad, 3 C_local)
    tp = qkv.shape[0] // b
    q3 = qkv.reshape(b, tp, -1)[:, :t]
    o = attention(q3)  # (B, T, C_local)
    if tp != t:
        o = torch.nn.functional.pad(o, (0, 0, 0, tp - t))
    x_r = row_parallel(o.reshape(b * tp, -1), attn.proj.weight, attn.proj.bias, ls1, res, sp)
    h2, res2 = layer_norm_residual(x_r, blk.norm2.weight, blk.norm2.bias, blk.norm2.eps)
    fc1 = getattr(mlp, "fc1", None)
    fc2 = getattr(mlp, "fc2", None)
    if fc1 is None or fc2 is None:
        raise NotImplementedError("sequence-parallel blocks support the GELU MLP (fc1 / fc2)")
    return mlp_parallel(h2, fc1.weight, fc1.bias, fc2.weight, fc2.bias, ls2, res2, sp)


def mark_partial_params(blocks: list[nn.Module], group: Any) -> int:
    """Mark the per-token-shard parameters (norms, LayerScale) whose gradients need a TP sum. The
    mark is kept on the owning module, which survives FSDP's replacement of its parameters."""
    count = 0
    for blk in blocks:
        for name in ("norm1", "norm2", "ls1", "ls2"):
            mod = getattr(blk, name, None)
            if mod is None:
                continue
            mod._sp_partial_group = group  # type: ignore[attr-defined]
            count += sum(1 for _ in mod.parameters(recurse=False))
    return count


def mark_post_gather_params(modules: list[nn.Module], group: Any) -> int:
    """Mark every parameter of modules that run after the final gather on this rank's slice of the
    batch: each rank's gradient covers its samples only and needs the TP sum."""
    count = 0
    for mod in modules:
        for m in mod.modules():
            if getattr(m, "_sp_partial_group", None) is None:
                m._sp_partial_group = group  # type: ignore[attr-defined]
                count += sum(1 for _ in m.parameters(recurse=False))
    return count


def _partial(module: nn.Module) -> list[tuple[Any, nn.Parameter]]:
    seen: set[int] = set()
    out = []
    for m in module.modules():
        grp = getattr(m, "_sp_partial_group", None)
        if grp is None:
            continue
        for p in m.parameters(recurse=False):
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                out.append((grp, p))
    return out


def partial_params(module: nn.Module) -> list[nn.Parameter]:
    return [p for _, p in _partial(module)]


@torch.no_grad()
def sync_partial_grads(module: nn.Module) -> int:
    """Sum the sequence-parallel partial gradients over their TP group (one all-reduce per group)."""
    groups: dict[int, tuple[Any, list[torch.Tensor]]] = {}
    for grp, p in _partial(module):
        g = getattr(p, "main_grad", None)
        if g is None:
            g = p.grad
        if g is None:
            continue
        to_local = getattr(g, "to_local", None)  # a data-parallel shard (FSDP2): its local part
        groups.setdefault(id(grp), (grp, []))[1].append(to_local() if to_local is not None else g)
    for grp, grads in groups.values():
        if dist.get_world_size(grp) == 1:
            continue
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        dist.all_reduce(flat, group=grp)
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n
    return sum(len(v[1]) for v in groups.values())
