"""A whole training step (forward, backward, grad clip, AdamW, schedule) captured in one CUDA graph.

The reference runs every step eagerly from Python: ~800 kernel launches per ViT-L MAE step, each
with autograd and dispatcher overhead on the host. Here the step is recorded once and replayed, so
the host issues a single graph launch per step and the device never waits for Python.

What makes the step capturable:

* `FlatParameters` packs every trainable parameter into one flat fp32 buffer (64-element aligned
  slots) with a flat fp32 gradient buffer. Each parameter gets `main_grad` (its slice of the
  gradient buffer) and, for matrices, `_mia_shadow` (a bf16 copy). Native backward kernels
  accumulate weight gradients straight into `main_grad`; gradients that arrive through autograd
  (parameters no native kernel owns) are folded in by a post-accumulate hook. The fused AdamW
  updates params and rewrites the bf16 shadows in the same pass, so GEMMs never cast weights.
* The learning-rate / weight-decay schedule is precomputed per step into a device table indexed by
  a device step counter, so nothing host-side changes between replays.
* Gradient clipping computes the global norm on the device and hands the clip coefficient to the
  AdamW kernel (no host synchronisation).
* Inputs are copied into static device buffers before each replay (from pinned host memory when
  the caller passes host tensors).

The first `eager_steps` calls run eagerly (they are real training steps and settle the allocator
and every lazily built table), the next call captures and replays. Metrics come back as static
device tensors; reading them is the caller's only synchronisation.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from typing import Any

import torch
import torch.nn as nn

from ..ops.optim import clip_coefficient, grad_sumsq
from .config import TrainerConfig
from .optimizer import lr_multiplier, weight_decay_at

_ALIGN = 64
# Data-parallel gradient paths: "allreduce" (NCCL all-reduce of the whole flat gradient, replicated
# AdamW), "p2p" (sharded optimizer over peer memory, engine/zero.py) and "nccl" (the same sharded
# layout over NCCL collectives).
DP_IMPLS = ("allreduce", "p2p", "nccl")


class FlatParameters:
    """Every trainable parameter of `module` as a view into flat fp32 param/grad buffers.

    Slots are `_ALIGN`-element aligned and the total is padded to a multiple of `world * _ALIGN`,
    so a sharded optimizer can split the buffer into equal, aligned, contiguous slices. With
    `bf16_region=True` the weights of Linear and convolution modules (whose only consumers run in
    bf16) are placed after everything else, starting at `bf16_begin`. The bf16 shadow buffer
    mirrors the fp32 layout element for element; parameters with `ndim >= shadow_min_dim` expose
    their slice of it as `_mia_shadow`. `allocate(numel, dtype) -> (tensor, peer pointers)` lets
    the caller place the buffers in peer-mapped memory.
    """

    def __init__(
        self,
        module: nn.Module,
        shadow_min_dim: int = 2,
        *,
        world: int = 1,
        bf16_region: bool = False,
        allocate: Callable[[int, torch.dtype], tuple[torch.Tensor, list[int] | None]] | None = None,
        groups: list[list[nn.Parameter]] | None = None,
    ) -> None:
        seen: set[int] = set()
        params: list[nn.Parameter] = []
        for p in module.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                params.append(p)
        if not params:
            raise ValueError("FlatParameters: nothing requires grad")
        gemm_weights: set[int] = set()
        if bf16_region:
            for m in module.modules():
                if isinstance(m, (nn.Linear, nn.modules.conv._ConvNd)) and isinstance(m.weight, nn.Parameter):
                    gemm_weights.add(id(m.weight))
        # groups: lists of bf16-region parameters that get segments of their own (in this order)
        grouped: list[list[nn.Parameter]] = []
        in_group: set[int] = set()
        for g in groups or []:
            members = [p for p in g if id(p) in gemm_weights and id(p) in seen and id(p) not in in_group]
            if members:
                grouped.append(members)
                in_group.update(id(p) for p in members)
        fp32_part = [p for p in params if id(p) not in gemm_weights]
        bf16_rest = [p for p in params if id(p) in gemm_weights and id(p) not in in_group]
        unit = _ALIGN * world
        device = params[0].device
        offsets: dict[int, int] = {}
        total = 0

        def place(p: nn.Parameter) -> None:
            nonlocal total
            offsets[id(p)] = total
            total += (p.numel() + _ALIGN - 1) // _ALIGN * _ALIGN

        for p in fp32_part:
            place(p)
        self.bf16_begin = total
        for p in bf16_rest:
            place(p)
        total = (total + unit - 1) // unit * unit
        self.segments: list[tuple[int, int]] = [(0, total)]
        for g in grouped:
            lo = total
            for p in g:
                place(p)
            total = (total + unit - 1) // unit * unit
            self.segments.append((lo, total))
        if total == 0:
            total = unit
            self.segments = [(0, unit)]
        if not bf16_region:
            self.bf16_begin = total  # no bf16 region: every parameter travels in fp32
        ordered = fp32_part + bf16_rest + [p for g in grouped for p in g]
        self.params = ordered
        self.offsets = [offsets[id(p)] for p in ordered]
        self.groups = grouped
        self.total = total
        self.world = world
        self.peers: dict[str, list[int]] | None = None
        if allocate is None:
            self.data = torch.zeros(total, dtype=torch.float32, device=device)
            self.grad = torch.zeros(total, dtype=torch.float32, device=device)
            self.shadow = torch.zeros(total, dtype=torch.bfloat16, device=device)
        else:
            self.data, pd = allocate(total, torch.float32)
            self.grad, pg = allocate(total, torch.float32)
            self.shadow, ps = allocate(total, torch.bfloat16)
            if pd is not None:
                self.peers = {"data": pd, "grad": pg, "shadow": ps}
        params = ordered
        self._hooks = []
        with torch.no_grad():
            for p, off in zip(params, self.offsets, strict=True):
                n = p.numel()
                view = self.data[off:off + n].view_as(p)
                view.copy_(p.data)
                p.data = view
                p.main_grad = self.grad[off:off + n].view_as(p)  # type: ignore[attr-defined]
                sview = self.shadow[off:off + n].view_as(p)
                sview.copy_(view)
                if p.ndim >= shadow_min_dim:
                    p._mia_shadow = sview  # type: ignore[attr-defined]
                self._hooks.append(p.register_post_accumulate_grad_hook(_fold_into_main_grad))
        self.numel = sum(p.numel() for p in params)

    def zero_grad(self) -> None:
        self.grad.zero_()

    @torch.no_grad()
    def refresh_shadows(self) -> None:
        """Re-derive the bf16 copies from the fp32 params (after loading weights)."""
        self.shadow.copy_(self.data)

    def release(self) -> None:
        for h in self._hooks:
            h.remove()
        for p in self.params:
            for attr in ("main_grad", "_mia_shadow"):
                if hasattr(p, attr):
                    delattr(p, attr)
        if self.peers is not None:  # peer-mapped buffers are about to be freed: give params their own memory
            with torch.no_grad():
                for p in self.params:
                    p.data = p.data.clone()


def _fold_into_main_grad(p: torch.Tensor) -> None:
    if p.grad is not None and getattr(p, "main_grad", None) is not None:
        p.main_grad.add_(p.grad)  # type: ignore[attr-defined]
        p.grad = None


class DeviceSchedule:
    """Per-step (lr, weight_decay, beta1, beta2) for every param group, as a device table."""

    def __init__(self, optimizer: torch.optim.Optimizer, config: TrainerConfig, start_step: int = 0) -> None:
        device = next(p.device for g in optimizer.param_groups for p in g["params"])
        steps = config.max_steps + 1
        table = torch.empty((steps, len(optimizer.param_groups), 4), dtype=torch.float32)
        for s in range(steps):
            mult = lr_multiplier(s, config)
            wd = weight_decay_at(s, config)
            for gi, group in enumerate(optimizer.param_groups):
                base_lr = group.get("initial_lr", group["lr"])
                b1, b2 = group["betas"]
                table[s, gi, 0] = base_lr * mult
                table[s, gi, 1] = wd * group.get("wd_multiplier", 1.0)
                table[s, gi, 2] = b1
                table[s, gi, 3] = b2
        self.table = table.to(device)
        self.counter = torch.tensor([start_step], dtype=torch.int64, device=device)
        self.current = torch.empty((len(optimizer.param_groups), 4), dtype=torch.float32, device=device)
        self.last_index = steps - 1

    def advance(self) -> torch.Tensor:
        """Load this step's row into `current`, then move the counter on (clamped at the end)."""
        idx = self.counter.clamp(max=self.last_index)
        self.current.copy_(self.table.index_select(0, idx)[0])
        self.counter.add_(1)
        return self.current


def _overlap_blocks(algorithm: nn.Module) -> list[nn.Module]:
    """The transformer blocks declared by the model and the algorithm, in module order."""
    from .activation_checkpoint import checkpointable_targets

    try:
        return checkpointable_targets(algorithm)
    except ValueError:
        return []


def _to_static(batch: Any, device: torch.device) -> Any:
    if isinstance(batch, torch.Tensor):
        return torch.empty(batch.shape, dtype=batch.dtype, device=device)
    if isinstance(batch, Mapping):
        return {k: _to_static(v, device) for k, v in batch.items()}
    if isinstance(batch, (list, tuple)):
        return type(batch)(_to_static(v, device) for v in batch)
    return batch


def _copy_into(static: Any, batch: Any) -> None:
    if isinstance(static, torch.Tensor):
        static.copy_(batch, non_blocking=True)
    elif isinstance(static, Mapping):
        for k in static:
            _copy_into(static[k], batch[k])
    elif isinstance(static, (list, tuple)):
        for s, b in zip(static, batch, strict=True):
            _copy_into(s, b)


class CapturedStep:
    """`step(batch) -> metrics` for one training step, replayed from a CUDA graph after warm-up."""

    def __init__(
        self,
        algorithm: nn.Module,
        optimizer: torch.optim.Optimizer,
        config: TrainerConfig,
        example_batch: Any,
        *,
        eager_steps: int = 2,
        start_step: int = 0,
        capture: bool = True,
        forward: Callable[[Any], dict[str, torch.Tensor]] | None = None,
        process_group: Any = None,
        dp_impl: str = "p2p",
        comm_timeout_ms: float = 10_000.0,
        overlap: bool = False,
        dp_wire: str = "bf16",
    ) -> None:
        if not hasattr(optimizer, "grad_scale"):
            raise TypeError("CapturedStep needs the fused optimizer (FusedAdamW)")
        if dp_impl not in DP_IMPLS:
            raise ValueError(f"dp_impl must be one of {DP_IMPLS}, got {dp_impl!r}")
        self.algorithm = algorithm
        self.optimizer = optimizer
        self.config = config
        self.device = next(algorithm.parameters()).device
        self.process_group = process_group
        self.world = 1
        if process_group is not None:
            import torch.distributed as dist

            self.world = dist.get_world_size(process_group)
        self.dp_impl = dp_impl if self.world > 1 else "allreduce"
        self.zero: Any = None
        if self.dp_impl == "allreduce":
            self.flat = FlatParameters(algorithm)
        else:
            from .zero import IpcBuffers, ShardedStep

            ipc = IpcBuffers(process_group, self.device) if self.dp_impl == "p2p" else None
            blocks = _overlap_blocks(algorithm) if overlap else []
            self.flat = FlatParameters(
                algorithm, world=self.world, bf16_region=config.precision == "bf16",
                allocate=ipc.allocate if ipc is not None else None,
                groups=[list(b.parameters()) for b in blocks],
            )
        self.schedule = DeviceSchedule(optimizer, config, start_step)
        optimizer.external_hyper = self.schedule.current  # type: ignore[attr-defined]
        if self.dp_impl != "allreduce":
            self.zero = ShardedStep(
                self.flat, optimizer, process_group, "p2p" if self.dp_impl == "p2p" else "nccl",
                config.grad_clip_norm, self.schedule.current, ipc=ipc, timeout_ms=comm_timeout_ms,
                wire_dtype=dp_wire,
            )
        # Reduce-scatter each block's weight gradients on a side stream as soon as the block's
        # backward has been issued (its input gradient is the last thing it computes).
        self._in_backward = False
        self._block_hooks: list[Any] = []
        self.comm_stream: torch.cuda.Stream | None = None
        if self.zero is not None and len(self.flat.segments) > 1:
            self.comm_stream = torch.cuda.Stream(self.device)
            segment_of = {}
            for gi, group in enumerate(self.flat.groups):
                for p in group:
                    segment_of[id(p)] = gi + 1
            for block in blocks:
                segs = {segment_of[id(p)] for p in block.parameters() if id(p) in segment_of}
                if len(segs) == 1:
                    self._block_hooks.append(block.register_full_backward_hook(self._make_hook(segs.pop())))
        self.static_batch = _to_static(example_batch, self.device)
        self._staging: Any = None
        self._copy_stream: torch.cuda.Stream | None = None
        self._prefetched = False
        self.static_metrics: dict[str, torch.Tensor] = {}
        self.eager_steps = eager_steps
        self.capture = capture
        self.calls = 0
        self.graph: torch.cuda.CUDAGraph | None = None
        self._forward = forward or algorithm
        self._autocast_dtype = torch.bfloat16 if config.precision == "bf16" else None

    def _make_hook(self, segment: int) -> Callable[..., None]:
        def hook(module: nn.Module, grad_input: Any, grad_output: Any) -> None:
            if not self._in_backward or self.comm_stream is None:
                return
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.device))
            self.comm_stream.wait_event(ready)
            with torch.cuda.stream(self.comm_stream):
                self.zero.reduce_segment(segment)

        return hook

    def _body(self) -> dict[str, torch.Tensor]:
        self.flat.zero_grad()
        self.schedule.advance()
        if self._autocast_dtype is not None:
            with torch.autocast("cuda", dtype=self._autocast_dtype):
                metrics = self._forward(self.static_batch)
        else:
            metrics = self._forward(self.static_batch)
        if self.zero is not None:
            self.zero.begin()
            if self.comm_stream is not None:  # the side stream joins this step's stream order
                self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        self._in_backward = True
        try:
            metrics["loss"].backward()
        finally:
            self._in_backward = False
        out = {k: v.detach() for k, v in metrics.items()}
        if self.zero is not None:
            if self.comm_stream is not None:
                torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
            norm = self.zero.finish()
            if self.config.grad_clip_norm is not None:
                out["grad_norm"] = norm
            return out
        if self.world > 1:
            import torch.distributed as dist

            # Data parallel: sum the flat gradient over ranks (NCCL, captured in the graph); the
            # 1/world average is folded into the scale the AdamW kernel applies.
            dist.all_reduce(self.flat.grad, group=self.process_group)
        inv_world = 1.0 / self.world
        if self.config.grad_clip_norm is not None:
            norm = grad_sumsq([self.flat.grad]).sqrt() * inv_world
            self.optimizer.grad_scale = clip_coefficient(norm, float(self.config.grad_clip_norm)) * inv_world
            out["grad_norm"] = norm
        elif self.world > 1:
            self.optimizer.grad_scale = torch.full((), inv_world, device=self.device)
        self.optimizer.step()
        return out

    def _store(self, out: dict[str, torch.Tensor]) -> None:
        for k, v in out.items():
            v = v.float().reshape(())
            if k not in self.static_metrics:
                self.static_metrics[k] = torch.zeros((), dtype=torch.float32, device=self.device)
            self.static_metrics[k].copy_(v)

    def _capture(self) -> None:
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._store(self._body())
        self.graph = graph

    def load_batch(self, batch: Any) -> None:
        _copy_into(self.static_batch, batch)

    def prefetch(self, batch: Any) -> None:
        """Start copying the next step's (pinned host) batch to the device on a side stream.

        The copy overlaps the step that is running; the next `__call__()` without a batch waits for
        it and moves it into the captured input buffers with one device-to-device copy.
        """
        if self._staging is None:
            self._staging = _to_static(batch, self.device)
            self._copy_stream = torch.cuda.Stream(self.device)
        self._copy_stream.wait_stream(torch.cuda.current_stream(self.device))  # staging is free again
        with torch.cuda.stream(self._copy_stream):
            _copy_into(self._staging, batch)
        self._prefetched = True

    def wait_prefetch(self) -> None:
        """Make the current stream wait for an outstanding `prefetch` copy."""
        if self._copy_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._copy_stream)

    def __call__(self, batch: Any | None = None) -> dict[str, torch.Tensor]:
        """Run one step on `batch` (host tensors are copied in; None reuses the static batch or
        takes the batch handed to `prefetch`)."""
        if batch is not None:
            self.load_batch(batch)
        elif self._prefetched:
            torch.cuda.current_stream(self.device).wait_stream(self._copy_stream)
            _copy_into(self.static_batch, self._staging)
            self._prefetched = False
        self.calls += 1
        if not self.capture or self.calls <= self.eager_steps:
            self._store(self._body())
            return self.static_metrics
        if self.graph is None:
            self._capture()
        self.graph.replay()
        return self.static_metrics

    def release(self) -> None:
        self.graph = None
        for h in self._block_hooks:
            h.remove()
        self._block_hooks = []
        if self.zero is not None:
            self.zero.gather_masters()
        self.flat.release()
        if self.zero is not None:
            self.zero.release()
        if hasattr(self.optimizer, "external_hyper"):
            del self.optimizer.external_hyper
