"""Step FLOPs measurement and windowed throughput (reference `src/engine/mfu.py:50-180`).

A step's FLOPs are measured once with `torch.utils.flop_counter.FlopCounterMode` on a real
forward+backward of the algorithm, not derived from `BaseModel.flops()`: masking, multi-crop and
decoders make a fixed formula wrong by several times. While counting, every op runs as PyTorch
math (`counting_kernels`), since the counter cannot see custom kernels. Gradients, RNG state and
buffers are restored afterwards so enabling the probe cannot change what a run trains.

`ThroughputMeter` times whole logging windows from a point right after the metric reduction
(which synchronises anyway) and discards the first window.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import torch
from torch.utils.flop_counter import FlopCounterMode

from ..layers.common.attention import counting_kernels


def measure_step_flops(algorithm: torch.nn.Module, batch: Any, autocast: Any) -> int:
    buffers = {name: buf.detach().clone() for name, buf in algorithm.named_buffers()}
    cpu_rng = torch.get_rng_state()
    cuda_rng = torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None
    try:
        with counting_kernels(algorithm), autocast():
            with FlopCounterMode(display=False) as counter:
                metrics = algorithm(batch)
                metrics["loss"].backward()
    finally:
        algorithm.zero_grad(set_to_none=True)
        torch.set_rng_state(cpu_rng)
        if cuda_rng is not None:
            torch.cuda.set_rng_state_all(cuda_rng)
        with torch.no_grad():
            for name, buf in algorithm.named_buffers():
                if name in buffers:
                    buf.copy_(buffers[name])
    return int(counter.get_total_flops())


@dataclass(frozen=True)
class Throughput:
    mfu: float | None
    tflops_per_s: float
    samples_per_s: float

    def as_metrics(self) -> dict[str, float]:
        out = {"tflops_per_s": self.tflops_per_s, "samples_per_s": self.samples_per_s}
        if self.mfu is not None:
            out["mfu"] = self.mfu
        return out


class ThroughputMeter:
    def __init__(self, step_flops: int, peak_flops: float | None, samples_per_step: int) -> None:
        self._step_flops = step_flops
        self._peak = peak_flops
        self._samples = samples_per_step
        self._last: float | None = None
        self._warmed = False

    def start(self) -> None:
        self._last = time.perf_counter()
        self._warmed = False

    def window(self, steps: int) -> Throughput | None:
        now = time.perf_counter()
        previous, self._last = self._last, now
        if previous is None or not self._warmed:
            self._warmed = True
            return None
        elapsed = now - previous
        rate = self._step_flops * steps / elapsed
        return Throughput(
            mfu=(rate / self._peak) if self._peak else None,
            tflops_per_s=rate / 1e12,
            samples_per_s=self._samples * steps / elapsed,
        )
