"""Cross-rank metric reduction and rank-0 logging (reference `src/utils/metrics.py:11-50`).

`reduce_metrics` differs from the reference in one respect: all metrics are stacked into ONE tensor
and reduced with ONE all-reduce and ONE device->host copy, instead of an all-reduce and an `.item()`
per metric. The values are the same global means.
"""

from __future__ import annotations

from pathlib import Path

import torch
import torch.distributed as dist

try:
    from torch.distributed.tensor import DTensor
except ImportError:  # pragma: no cover
    DTensor = ()  # type: ignore[assignment]


def reduce_metrics(metrics: dict[str, torch.Tensor | float]) -> dict[str, float]:
    """Average every metric over all ranks -> plain floats describing the global batch."""
    names = sorted(metrics)
    if not names:
        return {}
    values = []
    device = None
    for name in names:
        value = metrics[name]
        if isinstance(value, torch.Tensor):
            t = value.detach()
            if isinstance(t, DTensor):
                t = t.full_tensor()
            t = t.float().mean()
            device = device or t.device
        else:
            t = torch.tensor(float(value))
        values.append(t)
    device = device or torch.device("cpu")
    if dist.is_initialized() and dist.get_backend() == "nccl" and device.type == "cpu":
        device = torch.device("cuda", torch.cuda.current_device())
    stacked = torch.stack([v.to(device) for v in values])
    if dist.is_initialized():
        dist.all_reduce(stacked, op=dist.ReduceOp.SUM)
        stacked = stacked / dist.get_world_size()
    host = stacked.cpu().tolist()
    return dict(zip(names, host, strict=True))


class MetricLogger:
    """Prints `[prefix] step N k=v ...` and writes TensorBoard scalars, on the primary rank only."""

    def __init__(self, log_dir: Path | None = None, is_primary: bool = True) -> None:
        self._is_primary = is_primary
        self._writer = None
        if is_primary and log_dir is not None:
            try:
                from torch.utils.tensorboard import SummaryWriter

                self._writer = SummaryWriter(log_dir=str(log_dir))
            except ImportError:  # pragma: no cover - tensorboard is optional here
                self._writer = None

    def log(self, step: int, metrics: dict[str, float], prefix: str = "train") -> None:
        if not self._is_primary:
            return
        body = "  ".join(f"{name}={value:.6g}" for name, value in sorted(metrics.items()))
        print(f"[{prefix}] step {step}  {body}", flush=True)
        if self._writer is not None:
            for name, value in metrics.items():
                self._writer.add_scalar(f"{prefix}/{name}", value, step)

    def close(self) -> None:
        if self._writer is not None:
            self._writer.close()
            self._writer = None
