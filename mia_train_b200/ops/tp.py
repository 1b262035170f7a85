"""Collective GEMMs of sequence-parallel tensor parallelism: all-gather -> GEMM and GEMM -> reduce-scatter.

    ag_gemm(x_r, B)          -> (epi(gather(x)[M, K] . B^T), gather(x))    x_r: this rank's (S, K) rows
    gemm_rs(A, B)            -> residual_r + gamma * (sum over ranks of (A . B^T))[rows of r] + bias)

Two implementations of the same contract:

* `"fused"` -- one native kernel each (`csrc/tp_gemm.cu`): the gather or the scatter travels over
  NVLink peer memory from inside the tcgen05 GEMM, tile by tile, through a `TpWorkspace`.
* `"collective"` -- `torch.distributed` collectives around the plain GEMM (NCCL on GPUs, Gloo on
  CPUs); it is the baseline the fused kernels are measured against and the path CPU tests run.

The reference reaches tensor parallelism through `parallelize_module` with DTensor collectives
(`src/distributed/parallelize.py:16-26`) and ships no sequence-parallel plan.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from ._native import use_native
from .linear import ACT_DGELU, ACT_GELU, ACT_NONE, gelu_grad_reference, gelu_reference, gemm


def _gather_rows(x: torch.Tensor, group: Any) -> torch.Tensor:
    world = dist.get_world_size(group)
    if world == 1:
        return x.contiguous()
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, dim=0)


def _scatter_sum_rows(y: torch.Tensor, group: Any) -> torch.Tensor:
    """Sum over ranks, keep this rank's rows (reduce-scatter; all-reduce + slice where the backend has none)."""
    world = dist.get_world_size(group)
    if world == 1:
        return y
    rank = dist.get_rank(group)
    rows = y.shape[0] // world
    if dist.get_backend(group) == "nccl":
        out = torch.empty((rows, *y.shape[1:]), device=y.device, dtype=y.dtype)
        dist.reduce_scatter_tensor(out, y.contiguous(), group=group)
        return out
    y = y.contiguous()
    dist.all_reduce(y, group=group)
    return y[rank * rows:(rank + 1) * rows].contiguous()


class TpComm:
    """How the sequence-parallel layers of one TP group talk: fused kernels or collectives.

    The fused path's peer-memory workspace is created on first use and re-created (collectively:
    every rank of the group makes the same calls with the same shapes) when a call needs more
    room. Do that first call outside CUDA-graph capture.
    """

    def __init__(self, group: Any, impl: str = "fused", timeout_ms: float = 10_000.0) -> None:
        if impl not in ("fused", "collective"):
            raise ValueError(f"TP communication must be 'fused' or 'collective', got {impl!r}")
        self.group = group
        self.impl = impl
        self.timeout_ms = float(timeout_ms)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.workspace: Any | None = None

    def fused_on(self, x: torch.Tensor) -> bool:
        return self.impl == "fused" and use_native(x) and x.dtype == torch.bfloat16

    def workspace_for(self, rows: int, width: int, device: torch.device) -> Any:
        """A workspace for `rows` rows per rank of gathered / reduced matrices up to `width` columns."""
        ws = self.workspace
        if ws is not None and rows <= ws.max_rows and width <= ws.max_k and width <= ws.max_n:
            return ws
        from ..comm.tp_workspace import TpWorkspace

        if ws is not None:
            rows, width = max(rows, ws.max_rows), max(width, ws.max_k, ws.max_n)
            ws.release()
        self.workspace = TpWorkspace(self.group, device, rows, width, width, self.timeout_ms)
        return self.workspace

    def release(self) -> None:
        if self.workspace is not None:
            self.workspace.release()
            self.workspace = None


def ag_gemm(
    comm: TpComm,
    x: torch.Tensor,
    w: torch.Tensor,
    *,
    b_kmajor: bool = True,
    bias: torch.Tensor | None = None,
    act: int = ACT_NONE,
    aux: torch.Tensor | None = None,
    want_pre: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """(out (M, N), gathered x (M, K), pre-activation (M, N) when `want_pre` and act is GELU)."""
    s, k = x.shape
    m = s * comm.world
    n = w.shape[0] if b_kmajor else w.shape[1]
    if comm.fused_on(x):
        out = torch.empty((m, n), device=x.device, dtype=torch.bfloat16)
        full = torch.empty((m, k), device=x.device, dtype=torch.bfloat16)
        pre = torch.empty((m, n), device=x.device, dtype=torch.bfloat16) if (want_pre and act == ACT_GELU) else None
        ws = comm.workspace_for(s, k, x.device)
        ws.ag_gemm(x.contiguous(), w.contiguous(), out, full, bias, aux, pre, b_kmajor, act)
        return out, full, pre
    full = _gather_rows(x, comm.group)
    if use_native(full):
        pre = torch.empty((m, n), device=x.device, dtype=x.dtype) if (want_pre and act == ACT_GELU) else None
        out = gemm(full, w, b_kmajor=b_kmajor, out_dtype=x.dtype, bias=bias, act=act, aux=aux, aux_out=pre)
        return out, full, pre
    wm = w if b_kmajor else w.t()
    acc = full.float() @ wm.float().t()
    if bias is not None:
        acc = acc + bias.float()
    pre = None
    if act == ACT_GELU:
        pre = acc.to(x.dtype) if want_pre else None
        acc = gelu_reference(acc)
    elif act == ACT_DGELU:
        acc = acc * gelu_grad_reference(aux)
    return acc.to(x.dtype), full, pre


def gemm_rs(
    comm: TpComm,
    a: torch.Tensor,
    w: torch.Tensor,
    *,
    b_kmajor: bool = True,
    bias: torch.Tensor | None = None,
    gamma: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    want_pre: bool = False,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """(residual + gamma * (reduce-scatter(a . w^T) + bias), pre = reduced + bias when `want_pre`)."""
    m = a.shape[0]
    if m % comm.world:
        raise ValueError(f"{m} rows are not divisible by the TP size {comm.world}")
    s = m // comm.world
    n = w.shape[0] if b_kmajor else w.shape[1]
    if comm.fused_on(a):
        out = torch.empty((s, n), device=a.device, dtype=torch.bfloat16)
        pre = torch.empty((s, n), device=a.device, dtype=torch.bfloat16) if want_pre else None
        res = residual.contiguous() if residual is not None else None
        ws = comm.workspace_for(s, n, a.device)
        ws.gemm_rs(a.contiguous(), w.contiguous(), out, bias, gamma, res, pre, b_kmajor)
        return out, pre
    if use_native(a):
        part = gemm(a.contiguous(), w, b_kmajor=b_kmajor, out_dtype=torch.bfloat16)
    else:
        wm = w if b_kmajor else w.t()
        part = (a.float() @ wm.float().t()).to(a.dtype)
    red = _scatter_sum_rows(part, comm.group).float()
    if bias is not None:
        red = red + bias.float()
    pre = red.to(a.dtype) if want_pre else None
    if gamma is not None:
        red = red * gamma.float()
    if residual is not None:
        red = red + residual.float()
    return red.to(a.dtype), pre
