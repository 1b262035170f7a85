"""Model FLOPs utilisation: FLOPs of one real training step, and throughput over logging windows.

Role of reference `src/engine/mfu.py:50-180`; the code is this framework's own.

The FLOPs of a step are counted once, at start-up, by running one real forward and backward of the
algorithm under `torch.utils.flop_counter.FlopCounterMode` -- masking, multi-crop and decoders make
a formula from the architecture alone wrong by several times. The native kernels are invisible to
the counter, so the probe runs under `counting_kernels`, which routes every op of the model through
its PyTorch formulation for the duration. The probe must not change training: a `_StateGuard`
snapshots the RNG streams and every buffer before it and puts them back after it, and gradients are
dropped.

`ThroughputMeter.window(steps)` is called at each logging step (right after the metric reduction,
which synchronises the device anyway) and converts the wall time since the previous call into
TFLOP/s, samples/s and MFU. The first window includes start-up work and is not reported.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import torch
from torch.utils.flop_counter import FlopCounterMode

from ..layers.common.attention import counting_kernels


class _StateGuard:
    """Restores RNG state and buffer contents of `module` on exit; clears its gradients."""

    def __init__(self, module: torch.nn.Module) -> None:
        self.module = module

    def __enter__(self) -> _StateGuard:
        self.saved_buffers = [(b, b.detach().clone()) for b in self.module.buffers()]
        self.cpu_rng = torch.random.get_rng_state()
        self.gpu_rng = torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None
        return self

    def __exit__(self, *exc: Any) -> None:
        self.module.zero_grad(set_to_none=True)
        torch.random.set_rng_state(self.cpu_rng)
        if self.gpu_rng is not None:
            torch.cuda.set_rng_state_all(self.gpu_rng)
        with torch.no_grad():
            for live, copy in self.saved_buffers:
                live.copy_(copy)


def measure_step_flops(algorithm: torch.nn.Module, batch: Any, autocast: Any) -> int:
    """FLOPs of one forward + backward of `algorithm` on `batch` (PyTorch math, state untouched)."""
    counter = FlopCounterMode(display=False)
    with _StateGuard(algorithm), counting_kernels(algorithm), autocast(), counter:
        algorithm(batch)["loss"].backward()
    return int(counter.get_total_flops())


@dataclass(frozen=True)
class Throughput:
    mfu: float | None
    tflops_per_s: float
    samples_per_s: float

    def as_metrics(self) -> dict[str, float]:
        metrics = {"tflops_per_s": self.tflops_per_s, "samples_per_s": self.samples_per_s}
        return metrics if self.mfu is None else {**metrics, "mfu": self.mfu}


class ThroughputMeter:
    """Throughput of whole logging windows (wall clock between consecutive `window` calls)."""

    def __init__(self, step_flops: int, peak_flops: float | None, samples_per_step: int) -> None:
        self.step_flops = step_flops
        self.peak_flops = peak_flops
        self.samples_per_step = samples_per_step
        self._mark: float | None = None
        self._windows = 0

    def start(self) -> None:
        self._mark, self._windows = time.perf_counter(), 0

    def window(self, steps: int) -> Throughput | None:
        now = time.perf_counter()
        began, self._mark = self._mark, now
        self._windows += 1
        if began is None or self._windows == 1:  # start-up window: not representative
            return None
        seconds = now - began
        flops_per_s = self.step_flops * steps / seconds
        return Throughput(
            mfu=flops_per_s / self.peak_flops if self.peak_flops else None,
            tflops_per_s=flops_per_s * 1e-12,
            samples_per_s=self.samples_per_step * steps / seconds,
        )
