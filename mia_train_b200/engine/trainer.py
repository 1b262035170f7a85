"""The training loop (reference `src/engine/trainer.py:33-364`).

Same order and semantics as the reference: seed, activation checkpointing before sharding,
parallelize, optimizer + schedule + DCP manager, loaders over the data-parallel plane, a metric
logger on rank 0; then per step data wait -> host-to-device copy -> forward under autocast ->
backward -> grad clip -> optimizer/scheduler step -> zero_grad, with backbone freeze/unfreeze,
`data_wait_frac(_max)`, windowed MFU/throughput, periodic checkpoints and validation, and a final
checkpoint when the last step is off cadence.

Additions:
* `algorithm.after_optimizer_step(step)` runs after every optimizer step (the reference never
  updates the DINOv3 teacher; `dinov3` uses this hook for its EMA).
* With the fused optimizer the grad-clip coefficient stays on the device and is applied inside the
  AdamW kernel; nothing in a step waits on the host.
* `nan_guard` stops the run when a logged loss is non-finite; `watchdog_seconds` dumps all thread
  stacks when one step takes longer than that.
* At every logging step (already a device synchronisation) the native kernels' error word is read:
  a bounded wait that ran out raises `DeviceWaitError` instead of training on partial results.
"""

from __future__ import annotations

import contextlib
import faulthandler
import itertools
import math
import sys
import threading
import time
from collections.abc import Iterator
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh
from torch.utils.data import DataLoader, DistributedSampler

from ..algorithms.base import BaseAlgorithm
from ..data.base import BaseDataset
from ..ops._native import raise_on_device_errors
from ..parallel.sequence_parallel import sync_partial_grads
from ..parallel.parallel_dims import ParallelDims
from ..parallel.parallelize import parallelize_algorithm, refresh_fsdp_grad_dtypes
from ..utils.device import move_to_device
from ..utils.hardware_flops import peak_flops
from ..utils.metrics import MetricLogger, reduce_metrics
from .activation_checkpoint import apply_activation_checkpointing
from .checkpoint import CheckpointManager
from .config import TrainerConfig
from .mfu import ThroughputMeter, measure_step_flops
from .optimizer import build_lr_scheduler, build_optimizer, clip_grad_norm_, is_stem
from .profiler import StepProfiler, annotate, current_rank, should_profile

_AUTOCAST = {"bf16": torch.bfloat16}


class NonFiniteLossError(RuntimeError):
    pass


class StepWatchdog:
    """Dumps every thread's stack to stderr if a step runs longer than `seconds` (0 disables)."""

    def __init__(self, seconds: float) -> None:
        self.seconds = seconds
        self._deadline: float | None = None
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.fired = 0

    def __enter__(self) -> StepWatchdog:
        if self.seconds > 0:
            self._thread = threading.Thread(target=self._run, daemon=True, name="step-watchdog")
            self._thread.start()
        return self

    def __exit__(self, *exc: Any) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=1.0)

    def arm(self) -> None:
        self._deadline = time.monotonic() + self.seconds if self.seconds > 0 else None

    def _run(self) -> None:
        while not self._stop.wait(min(1.0, self.seconds / 4)):
            deadline = self._deadline
            if deadline is not None and time.monotonic() > deadline:
                self.fired += 1
                print(f"[watchdog] a step exceeded {self.seconds:.0f} s; thread stacks follow", file=sys.stderr, flush=True)
                faulthandler.dump_traceback(file=sys.stderr, all_threads=True)
                self._deadline = None


class Trainer:
    def __init__(
        self,
        algorithm: BaseAlgorithm,
        train_dataset: BaseDataset,
        config: TrainerConfig,
        output_dir: Path,
        dims: ParallelDims | None = None,
        mesh: DeviceMesh | None = None,
        val_dataset: BaseDataset | None = None,
        device: torch.device | None = None,
    ) -> None:
        self.config = config
        self.dims = dims or ParallelDims()
        self.mesh = mesh
        self.output_dir = Path(output_dir)
        self.device = device or torch.device("cpu")
        torch.manual_seed(config.seed)
        if config.activation_checkpointing:
            apply_activation_checkpointing(algorithm)
        algorithm = algorithm.to(self.device)
        self.graph_mode = config.step_mode == "graph"
        if self.graph_mode:
            self._check_graph_mode()
        if mesh is not None and not self.graph_mode:
            parallelize_algorithm(algorithm, mesh, self.dims)
        elif self.graph_mode and dist.is_initialized() and dist.get_world_size() > 1:
            for t in list(algorithm.parameters()) + list(algorithm.buffers()):  # identical replicas
                dist.broadcast(t.data, src=0)
        self.graph_step: Any = None
        self.algorithm = algorithm
        self.optimizer = build_optimizer(self.algorithm, config)
        self.scheduler = build_lr_scheduler(self.optimizer, config)
        self.checkpoints = CheckpointManager(self.algorithm, self.optimizer, self.output_dir / "checkpoints")
        dp_rank = self.dims.dp_rank(mesh) if mesh is not None else 0
        loader_args = {
            "batch_size": config.batch_size,
            "rank": dp_rank,
            "world_size": self.dims.dp_world_size,
            "num_workers": config.num_workers,
            "persistent_workers": config.persistent_workers,
            "prefetch_factor": config.prefetch_factor,
        }
        self.train_loader = train_dataset.build_dataloader(**loader_args)
        self.val_loader = val_dataset.build_dataloader(shuffle=False, **loader_args) if val_dataset else None
        self.is_primary = not dist.is_initialized() or dist.get_rank() == 0
        self.logger = MetricLogger(log_dir=self.output_dir / "tensorboard", is_primary=self.is_primary)

    def _check_graph_mode(self) -> None:
        problems = []
        if self.device.type != "cuda":
            problems.append("a CUDA device")
        if self.config.fused_optimizer == "off":
            problems.append("the fused optimizer (fused_optimizer != 'off')")
        if self.dims.tp > 1:
            problems.append("tp = 1 (tensor parallelism runs eagerly)")
        if self.config.freeze_backbone_steps > 0:
            problems.append("no backbone freeze (the captured step cannot change requires_grad)")
        if problems:
            raise ValueError("step_mode = 'graph' needs " + ", ".join(problems))

    def _build_graph_step(self, example: Any, start_step: int) -> Any:
        from .graph_step import CapturedStep

        group = dist.group.WORLD if dist.is_initialized() and dist.get_world_size() > 1 else None
        step = CapturedStep(self.algorithm, self.optimizer, self.config, example, start_step=start_step,
                            process_group=group, dp_impl=self.config.graph_dp)
        if step.zero is not None:
            step.zero.import_state(self.optimizer)
        return step

    def _save(self, step: int) -> None:
        if self.graph_step is not None and self.graph_step.zero is not None:
            self.graph_step.zero.export_state(self.optimizer)
        self.checkpoints.save(step)
        if self.graph_step is not None and self.graph_step.zero is not None:
            self.optimizer.state.clear()

    def _autocast(self) -> Any:
        dtype = _AUTOCAST.get(self.config.precision)
        if dtype is None:
            return contextlib.nullcontext()
        return torch.autocast(self.device.type, dtype=dtype)

    def _backbone_parameters(self) -> list[tuple[str, torch.nn.Parameter]]:
        return [(n, p) for n, p in self.algorithm.model.named_parameters() if not is_stem(n)]

    def _set_backbone_frozen(self, frozen: bool) -> None:
        params = self._backbone_parameters()
        for _, p in params:
            p.requires_grad_(not frozen)
        refresh_fsdp_grad_dtypes(self.algorithm)
        if self.is_primary:
            count = sum(p.numel() for _, p in params)
            print(
                f"[freeze] {'froze' if frozen else 'unfroze'} {len(params)} backbone tensors ({count / 1e6:.1f}M params)",
                flush=True,
            )

    def _peak_flops(self) -> tuple[float | None, str]:
        if self.config.peak_tflops is not None:
            return self.config.peak_tflops * 1e12, ""
        if self.device.type != "cuda":
            return None, f"no peak-FLOPS figure for device type {self.device.type!r}"
        return peak_flops(torch.cuda.get_device_name(self.device), self.config.precision)

    def _build_throughput_meter(self, batch: Any) -> ThroughputMeter:
        peak, reason = self._peak_flops()
        if peak is None and self.is_primary:
            print(f"[mfu] utilization not reported: {reason}", flush=True)
        step_flops = measure_step_flops(self.algorithm, batch, self._autocast)
        if self.is_primary:
            note = f"{peak / 1e12:.1f} TFLOP/s peak" if peak else "peak unknown"
            print(f"[mfu] measured {step_flops / 1e12:.3f} TFLOP per step per rank, {note}", flush=True)
        return ThroughputMeter(step_flops, peak, self.config.batch_size * self.dims.dp_world_size)

    def _endless_batches(self, loader: DataLoader, start_epoch: int = 0) -> Iterator[Any]:
        epoch = start_epoch
        while True:
            if isinstance(loader.sampler, DistributedSampler):
                loader.sampler.set_epoch(epoch)
            yield from loader
            epoch += 1

    def _clip(self) -> torch.Tensor:
        """Global grad norm; with the fused optimizer the clip is deferred into the AdamW kernel."""
        params = [p for p in self.algorithm.parameters() if p.grad is not None]
        fused = hasattr(self.optimizer, "grad_scale")
        if fused and params and all(type(p.grad) is torch.Tensor for p in params):
            from ..ops.optim import clip_coefficient, grad_sumsq

            norm = grad_sumsq([p.grad for p in params]).sqrt()
            self.optimizer.grad_scale = clip_coefficient(norm, float(self.config.grad_clip_norm))
            return norm
        return clip_grad_norm_(params, float(self.config.grad_clip_norm))

    def train(self) -> int:
        step = self.checkpoints.load_latest()
        resumed_from = step
        for _ in range(step):
            self.scheduler.step()
        batches = self._endless_batches(self.train_loader, start_epoch=step)
        self.algorithm.train()
        frozen = step < self.config.freeze_backbone_steps
        if frozen:
            self._set_backbone_frozen(True)
        meter: ThroughputMeter | None = None
        if self.config.measure_mfu and step < self.config.max_steps:
            probe = move_to_device(next(batches), self.device)
            batches = itertools.chain([probe], batches)
            meter = self._build_throughput_meter(probe)
            meter.start()
        logged_at = step
        data_seconds = 0.0
        window_start = time.perf_counter()
        profiling = self.config.profile and should_profile(current_rank(), self.config.profile_all_ranks)
        with StepProfiler(
            self.output_dir,
            start_step=self.config.profile_start_step,
            active=self.config.profile_steps,
            profile_memory=self.config.profile_memory,
            enabled=profiling,
        ) as profiler, StepWatchdog(self.config.watchdog_seconds) as watchdog:
            while step < self.config.max_steps:
                watchdog.arm()
                t0 = time.perf_counter()
                with annotate("data_wait"):
                    raw = next(batches)
                data_seconds += time.perf_counter() - t0
                if self.graph_mode:
                    if self.graph_step is None:
                        self.graph_step = self._build_graph_step(raw, step)
                    with annotate("graph_step"):
                        metrics = dict(self.graph_step(raw))
                    self.scheduler.step()
                else:
                    with annotate("h2d"):
                        batch = move_to_device(raw, self.device)
                    with annotate("forward"), self._autocast():
                        metrics = self.algorithm(batch)
                    with annotate("backward"):
                        metrics["loss"].backward()
                        # sequence-parallel TP: norm / LayerScale (and decoder, when the batch is
                        # split over the TP ranks) gradients are per-rank partial sums
                        sync_partial_grads(self.algorithm)
                    if self.config.grad_clip_norm is not None:
                        with annotate("grad_clip"):
                            metrics["grad_norm"] = self._clip()
                    with annotate("optimizer"):
                        self.optimizer.step()
                        self.scheduler.step()
                        self.optimizer.zero_grad(set_to_none=True)
                step += 1
                self.algorithm.after_optimizer_step(step)
                if frozen and step >= self.config.freeze_backbone_steps:
                    self._set_backbone_frozen(False)
                    frozen = False
                if step % self.config.log_every == 0:
                    logged = reduce_metrics(metrics)
                    # reduce_metrics synchronised the device: read the kernels' error word here, so a
                    # wait that timed out (a lost peer, a stuck pipeline) stops the run instead of
                    # letting AdamW apply partial gradients.
                    raise_on_device_errors(self.device)
                    if self.config.nan_guard and not math.isfinite(logged.get("loss", 0.0)):
                        raise NonFiniteLossError(f"loss became {logged['loss']} at step {step}")
                    logged["lr"] = float(self.scheduler.get_last_lr()[0])
                    now = time.perf_counter()
                    stalled = data_seconds / max(now - window_start, 1e-9)
                    logged["data_wait_frac"] = stalled
                    if dist.is_initialized():
                        worst = torch.tensor(stalled, device=self.device if dist.get_backend() == "nccl" else "cpu")
                        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
                        logged["data_wait_frac_max"] = float(worst.item())
                    data_seconds, window_start = 0.0, now
                    if meter is not None:
                        window = meter.window(step - logged_at)
                        if window is not None:
                            logged.update(window.as_metrics())
                    logged_at = step
                    self.logger.log(step, logged)
                if self.config.checkpoint_every and step % self.config.checkpoint_every == 0:
                    self._save(step)
                if self.config.val_every and step % self.config.val_every == 0:
                    self.logger.log(step, self.validate(), prefix="val")
                    self.algorithm.train()
                    data_seconds, window_start = 0.0, time.perf_counter()
                profiler.step()
        if self.config.checkpoint_every and step > resumed_from and step % self.config.checkpoint_every != 0:
            self._save(step)
        if self.graph_step is not None:
            self.graph_step.release()
            self.graph_step = None
        raise_on_device_errors(self.device)
        self.logger.close()
        return step

    def validate(self) -> dict[str, float]:
        if self.val_loader is None:
            raise ValueError("Trainer was constructed without a val_dataset")
        self.algorithm.eval()
        totals: dict[str, float] = {}
        count = 0
        with torch.no_grad():
            for batch in self.val_loader:
                with self._autocast():
                    metrics = self.algorithm.validation_step(move_to_device(batch, self.device))
                for name, value in reduce_metrics(metrics).items():
                    totals[name] = totals.get(name, 0.0) + value
                count += 1
        return {name: total / max(1, count) for name, total in totals.items()}
