"""Sharded data-parallel optimizer step (gradients reduce-scattered, AdamW on a shard, params gathered).

Every rank keeps the whole model (a ViT-L is 1.3 GB of fp32 parameters against 180 GB of HBM), so
forward and backward need no parameter collectives at all. After backward, rank r owns the r-th
contiguous slice of the flat parameter buffer:

1. reduce-scatter: rank r sums slice r of every rank's flat gradient (with the p2p implementation
   the gradients travel in bf16 by default -- each rank rounds its fp32 gradient into a peer-mapped
   bf16 buffer and the owner sums the copies in fp32; `wire_dtype="fp32"` reads the fp32 values),
2. the global gradient norm is exchanged and turned into the clip coefficient (times 1/world),
3. AdamW updates slice r only (exp_avg / exp_avg_sq exist only for the owned slice, so optimizer
   memory is 1/world of the unsharded optimizer),
4. all-gather: every rank receives the other slices. Matrices consumed by GEMMs and convolutions
   (the bf16 region of `FlatParameters`) travel as their bf16 values -- under bf16 compute that is
   all any consumer reads -- and the receiver rebuilds its fp32 copy from them; everything else
   travels in fp32. The owner keeps the exact fp32 master of its slice.

Two implementations of the same layout:

* `"p2p"` -- three native kernels over CUDA-IPC peer memory (`csrc/comm.cu`): the
  reduce-scatter reads every peer's gradient slice over NVLink with 16-byte loads, the norm
  exchange is one CTA, the all-gather pushes the owned slice into every peer with 16-byte stores
  and refreshes the received slices locally; barriers are flag words with bounded waits.
* `"nccl"` -- `reduce_scatter_tensor` / `all_reduce` / `all_gather_into_tensor` on the same flat
  buffers (fp32 all-gather of the whole slice), kept as the baseline the fused path is compared to.

The reference reaches the same end through FSDP2 (`src/distributed/parallelize.py:29-57`), which
all-gathers fp32 parameters per unit in forward and backward and reduce-scatters fp32 gradients.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from ..comm.ipc import IpcBuffers, all_gather_cpu  # noqa: F401  (IpcBuffers re-exported)
from ..ops._native import native
from ..ops.optim import adamw_step, clip_coefficient, grad_sumsq

IMPLS = ("p2p", "nccl")


class ShardedStep:
    """Steps 1-4 above for a `FlatParameters` built with `world` (and optionally segments).

    The flat buffer is cut into the segments of `flat.segments`; rank r owns the r-th slice of
    every segment. `reduce_segment(i)` can run as soon as segment i's gradients are final (the
    graph step calls it from block backward hooks on a side stream, so the reduce-scatter of late
    layers overlaps the backward of earlier ones); `finish()` reduces what is left, exchanges the
    norm, runs AdamW on the owned slices and all-gathers every segment.
    """

    def __init__(
        self,
        flat: Any,
        optimizer: torch.optim.Optimizer,
        group: Any,
        impl: str,
        max_norm: float | None,
        hyper: torch.Tensor,
        ipc: IpcBuffers | None = None,
        timeout_ms: float = 10_000.0,
        overlap_blocks: int = 64,
        wire_dtype: str = "bf16",
    ) -> None:
        if impl not in IMPLS:
            raise ValueError(f"sharded step impl must be one of {IMPLS}, got {impl!r}")
        self.flat = flat
        self.group = group
        self.impl = impl
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_norm = float(max_norm) if max_norm is not None else 0.0
        self.timeout_ms = timeout_ms
        self.hyper = hyper
        dev = flat.data.device
        # owned slice of every segment: (segment lo, slice length, offset of the slice in the moments)
        self.owned: list[tuple[int, int, int]] = []
        moment_off = 0
        for lo, hi in flat.segments:
            sl = (hi - lo) // self.world
            self.owned.append((lo, sl, moment_off))
            moment_off += sl
        self.owned_numel = moment_off
        group_of = {id(p): gi for gi, g in enumerate(optimizer.param_groups) for p in g["params"]}
        eps = {g["eps"] for g in optimizer.param_groups}
        if len(eps) != 1:
            raise ValueError("the sharded AdamW needs one eps for all param groups")
        self.eps = float(eps.pop())
        self.exp_avg = torch.zeros(max(moment_off, 1), dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(max(moment_off, 1), dtype=torch.float32, device=dev)
        params, grads, m, v, steps, gidx, shadows = [], [], [], [], [], [], []
        self.slices: list[tuple[Any, int, int, int]] = []  # (param, a, b, moment offset of a)
        for p, off in zip(flat.params, flat.offsets, strict=True):
            if id(p) not in group_of:
                raise ValueError("every flat parameter must belong to an optimizer param group")
            for lo, sl, mo in self.owned:
                own_lo = lo + self.rank * sl
                a, b = max(off, own_lo), min(off + p.numel(), own_lo + sl)
                if a >= b:
                    continue
                ma = mo + (a - own_lo)
                params.append(flat.data[a:b])
                grads.append(flat.grad[a:b])
                m.append(self.exp_avg[ma:ma + (b - a)])
                v.append(self.exp_avg_sq[ma:ma + (b - a)])
                steps.append(torch.zeros((), dtype=torch.float32, device=dev))
                gidx.append(group_of[id(p)])
                shadows.append(flat.shadow[a:b])
                self.slices.append((p, a, b, ma))
        self._lists = (params, grads, m, v, steps, shadows)
        self._gidx = torch.tensor(gidx, dtype=torch.int32, device=dev)
        self.grad_scale = torch.ones((), dtype=torch.float32, device=dev)
        self.grad_norm = torch.zeros((), dtype=torch.float32, device=dev)
        self._own_grads = [flat.grad[lo + self.rank * sl: lo + (self.rank + 1) * sl] for lo, sl, _ in self.owned]
        self._reduced = [False] * len(self.owned)
        self._seq = 0
        if impl == "p2p":
            if ipc is None or flat.peers is None:
                raise ValueError("the p2p implementation needs FlatParameters allocated through IpcBuffers")
            self.ipc = ipc
            self.blocks = min(2 * torch.cuda.get_device_properties(dev).multi_processor_count,
                              int(native().comm_max_blocks()))
            self.overlap_blocks = max(1, min(overlap_blocks, self.blocks))
            # per-segment slices of the partial sums: the tail segment (0) uses the full grid
            grids = [self.blocks] + [self.overlap_blocks] * (len(self.owned) - 1)
            self._partial_off = [sum(grids[:i]) for i in range(len(grids))]
            self._grids = grids
            self.partial = torch.zeros(sum(grids), dtype=torch.float32, device=dev)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
            _, self.flag_peers = ipc.allocate(int(native().comm_flag_bytes()) // 4, torch.int32)
            if wire_dtype not in ("bf16", "fp32"):
                raise ValueError(f"wire_dtype must be 'bf16' or 'fp32', got {wire_dtype!r}")
            self.wire_dtype = wire_dtype
            # bf16 wire format: each rank rounds its fp32 gradients into this peer-mapped buffer and
            # the owners sum the bf16 copies in fp32 (half the NVLink bytes of reading fp32)
            self.grad16_peers = ipc.allocate(flat.total, torch.bfloat16)[1] if wire_dtype == "bf16" else None

    # -- reduce-scatter -------------------------------------------------------------------------
    def begin(self) -> None:
        """Start of a step's gradient phase (before backward)."""
        self._reduced = [False] * len(self.owned)
        self._seq = 0

    def reduce_segment(self, i: int) -> None:
        """Reduce-scatter segment i on the current stream (its gradients must be final)."""
        if self._reduced[i]:
            return
        self._reduced[i] = True
        lo, sl, _ = self.owned[i]
        if self.impl == "p2p":
            grid = self._grids[i]
            part = self.partial[self._partial_off[i]:self._partial_off[i] + grid]
            # Segments reduced during backward use small CTAs (128 threads, no shared memory) so they
            # fit on an SM beside a GEMM CTA instead of displacing it.
            threads = 512 if i == 0 else 128
            if self.grad16_peers is not None:
                native().zero_reduce_scatter_bf16(self.flat.peers["grad"], self.grad16_peers, self.flag_peers, lo, sl,
                                                  part, self.epoch, self.rank, self.timeout_ms, self._seq, threads)
            else:
                native().zero_reduce_scatter(self.flat.peers["grad"], self.flag_peers, lo + self.rank * sl, sl, part,
                                             self.epoch, self.rank, self.timeout_ms, self._seq, threads)
        else:
            dist.reduce_scatter_tensor(self._own_grads[i], self.flat.grad[lo:lo + self.world * sl], group=self.group)
        self._seq += 1

    def finish(self) -> torch.Tensor:
        """Reduce the remaining segments, clip, AdamW on the owned slices, all-gather; returns the norm."""
        for i in range(len(self.owned) - 1, -1, -1):
            self.reduce_segment(i)
        params, grads, m, v, steps, shadows = self._lists
        if self.impl == "p2p":
            n = native()
            n.zero_norm_exchange(self.flag_peers, self.partial, self.epoch, self.rank, self.max_norm,
                                 self.grad_scale, self.grad_norm, self.timeout_ms)
            if params:
                adamw_step(params, grads, m, v, steps, self._gidx, self.hyper, self.eps, self.grad_scale, shadows)
            for seq, (lo, sl, _) in enumerate(self.owned):
                n.zero_all_gather(self.flat.peers["data"], self.flat.peers["shadow"], self.flag_peers, lo, sl,
                                  self.flat.bf16_begin, self.epoch, self.rank, self.blocks, self.timeout_ms, seq)
            n.zero_advance_epoch(self.epoch)
            return self.grad_norm
        sumsq = grad_sumsq(self._own_grads)
        dist.all_reduce(sumsq, group=self.group)
        norm = sumsq.sqrt() / self.world
        coef = clip_coefficient(norm, self.max_norm) if self.max_norm > 0 else torch.ones_like(norm)
        self.grad_scale.copy_(coef / self.world)
        self.grad_norm.copy_(norm)
        if params:
            adamw_step(params, grads, m, v, steps, self._gidx, self.hyper, self.eps, self.grad_scale, shadows)
        for lo, sl, _ in self.owned:
            seg = self.flat.data[lo:lo + self.world * sl]
            dist.all_gather_into_tensor(seg, seg[self.rank * sl:(self.rank + 1) * sl], group=self.group)
        self.flat.shadow.copy_(self.flat.data)
        return self.grad_norm

    def step(self) -> torch.Tensor:
        """Whole gradient phase after backward (no overlap)."""
        self.begin()
        return self.finish()

    @torch.no_grad()
    def gather_masters(self) -> None:
        """Make every rank's fp32 copy exact (the bf16 region is bf16-rounded off the owner)."""
        for lo, sl, _ in self.owned:
            seg = self.flat.data[lo:lo + self.world * sl]
            dist.all_gather_into_tensor(seg, seg[self.rank * sl:(self.rank + 1) * sl].clone(), group=self.group)

    @torch.no_grad()
    def _full_moments(self) -> dict[str, torch.Tensor]:
        """Whole-buffer moments (flat layout) gathered from every rank's owned slices."""
        dev = self.flat.data.device
        out = {}
        for name, mine in (("exp_avg", self.exp_avg), ("exp_avg_sq", self.exp_avg_sq)):
            full = torch.zeros(self.flat.total, dtype=torch.float32, device=dev)
            for lo, sl, mo in self.owned:
                seg = full[lo:lo + self.world * sl]
                dist.all_gather_into_tensor(seg, mine[mo:mo + sl].contiguous(), group=self.group)
            out[name] = full
        return out

    @torch.no_grad()
    def export_state(self, optimizer: torch.optim.Optimizer) -> None:
        """Write whole-parameter AdamW state (torch layout) into `optimizer.state` on every rank."""
        self.gather_masters()
        full = self._full_moments()
        dev = self.flat.data.device
        step = self._lists[4][0].detach().clone() if self._lists[4] else torch.zeros((), device=dev)
        dist.broadcast(step, src=dist.get_global_rank(self.group, 0) if self.group is not None else 0, group=self.group)
        for p, off in zip(self.flat.params, self.flat.offsets, strict=True):
            n = p.numel()
            optimizer.state[p] = {
                "step": step.clone(),
                "exp_avg": full["exp_avg"][off:off + n].view_as(p).clone(),
                "exp_avg_sq": full["exp_avg_sq"][off:off + n].view_as(p).clone(),
            }

    @torch.no_grad()
    def import_state(self, optimizer: torch.optim.Optimizer) -> bool:
        """Load the owned slices' moments from whole-parameter state in `optimizer.state` (if any)."""
        offsets = {id(p): off for p, off in zip(self.flat.params, self.flat.offsets, strict=True)}
        found = False
        steps = self._lists[4]
        for i, (p, a, b, ma) in enumerate(self.slices):
            state = optimizer.state.get(p)
            if not state or "exp_avg" not in state:
                continue
            found = True
            off = offsets[id(p)]
            self.exp_avg[ma:ma + (b - a)].copy_(state["exp_avg"].reshape(-1)[a - off:b - off])
            self.exp_avg_sq[ma:ma + (b - a)].copy_(state["exp_avg_sq"].reshape(-1)[a - off:b - off])
            steps[i].copy_(state["step"])
        optimizer.state.clear()  # the shards are the live state now
        return found

    def release(self) -> None:
        if self.impl == "p2p":
            self.ipc.release()
