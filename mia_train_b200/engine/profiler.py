"""Step profiling and trace summaries (reference `src/engine/profiler.py:53-315`).

* `StepProfiler` wraps `torch.profiler` (CPU + CUDA, shapes recorded, optional memory) with a
  schedule that skips `start_step` steps of this process, warms up one and records `active`, and
  writes a TensorBoard/Chrome trace into `<run>/profile/`.
* `annotate(name)` is a `record_function` range plus an NVTX range (visible to Nsight tools).
* `python -m mia_train_b200.engine.profiler RUN` summarises the newest trace under a run: GPU busy
  vs idle (union of device intervals), annotated regions (host and device), host time blocked in
  synchronize calls, and the slowest kernels.
* `RegionTimer` (new) times named regions on the device with CUDA events, for per-region
  device-time without a profiler attached.
"""

from __future__ import annotations

import argparse
import contextlib
import gzip
import json
from collections import defaultdict
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist


class StepProfiler:
    def __init__(
        self, output_dir: Path, start_step: int, active: int, profile_memory: bool = False, enabled: bool = True
    ) -> None:
        self._enabled = enabled
        self._profiler: Any = None
        self._trace_dir: Path | None = None
        if not enabled:
            return
        self._trace_dir = Path(output_dir) / "profile"
        self._trace_dir.mkdir(parents=True, exist_ok=True)
        activities = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            activities.append(torch.profiler.ProfilerActivity.CUDA)
        self._profiler = torch.profiler.profile(
            activities=activities,
            schedule=torch.profiler.schedule(skip_first=start_step, wait=0, warmup=1, active=active, repeat=1),
            on_trace_ready=torch.profiler.tensorboard_trace_handler(str(self._trace_dir)),
            record_shapes=True,
            profile_memory=profile_memory,
            with_stack=False,
        )

    def __enter__(self) -> StepProfiler:
        if self._profiler is not None:
            self._profiler.__enter__()
        return self

    def __exit__(self, *exc: Any) -> None:
        if self._profiler is not None:
            self._profiler.__exit__(*exc)
            self._profiler = None

    def step(self) -> None:
        if self._profiler is not None:
            self._profiler.step()

    @property
    def trace_dir(self) -> Path | None:
        return self._trace_dir if self._enabled else None


def should_profile(rank: int, all_ranks: bool) -> bool:
    return all_ranks or rank == 0


def current_rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


@contextlib.contextmanager
def annotate(name: str) -> Any:
    nvtx = torch.cuda.is_available() and not torch.cuda.is_current_stream_capturing()
    if nvtx:
        torch.cuda.nvtx.range_push(name)
    try:
        with torch.profiler.record_function(name):
            yield
    finally:
        if nvtx:
            torch.cuda.nvtx.range_pop()


class RegionTimer:
    """Accumulate device time per named region with CUDA events (no-op on CPU)."""

    def __init__(self, enabled: bool = True) -> None:
        self.enabled = enabled and torch.cuda.is_available()
        self._pending: list[tuple[str, Any, Any]] = []
        self.totals: dict[str, float] = defaultdict(float)

    @contextlib.contextmanager
    def region(self, name: str) -> Any:
        if not self.enabled:
            yield
            return
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self._pending.append((name, start, end))

    def collect(self) -> dict[str, float]:
        for name, start, end in self._pending:
            end.synchronize()
            self.totals[name] += start.elapsed_time(end)
        self._pending.clear()
        return dict(self.totals)


def find_trace(target: Path) -> Path:
    target = Path(target)
    if target.is_file():
        return target
    for candidate in (target / "profile", target):
        if candidate.is_dir():
            traces = sorted(candidate.glob("*.pt.trace.json*"))
            if traces:
                return max(traces, key=lambda p: p.stat().st_mtime)
    raise FileNotFoundError(
        f"no *.pt.trace.json under {target}; pass a run directory with a profile/ subdirectory or a "
        "trace file (a run writes one only with [trainer].profile = true)"
    )


def _events(path: Path) -> list[dict[str, Any]]:
    opener = gzip.open if path.suffix == ".gz" else open
    with opener(path, "rt") as handle:
        return list(json.load(handle)["traceEvents"])


def union_length(spans: list[tuple[float, float]]) -> float:
    """Total length covered by a set of (start, end) intervals."""
    if not spans:
        return 0.0
    spans = sorted(spans)
    total = 0.0
    cur_start, cur_end = spans[0]
    for s, e in spans[1:]:
        if s > cur_end:
            total += cur_end - cur_start
            cur_start, cur_end = s, e
        else:
            cur_end = max(cur_end, e)
    return total + cur_end - cur_start


def summarize(trace_path: Path) -> str:
    events = [e for e in _events(trace_path) if e.get("ph") == "X" and e.get("dur") is not None]
    cats: dict[str, list[dict[str, Any]]] = defaultdict(list)
    for e in events:
        cats[str(e.get("cat", "?"))].append(e)
    device = cats["kernel"] + cats["gpu_memcpy"] + cats["gpu_memset"]
    if not device:
        return f"{trace_path}\n\nNo GPU activity in this trace -- was the run on CPU?"
    steps = [e for e in events if str(e.get("name", "")).startswith("ProfilerStep")]
    n = len(steps) or 1
    first = min(e["ts"] for e in device)
    last = max(e["ts"] + e["dur"] for e in device)
    window_ms = (last - first) / 1000.0
    step_ms = sum(e["dur"] for e in steps) / 1000.0 / n if steps else window_ms / n
    busy_ms = union_length([(e["ts"], e["ts"] + e["dur"]) for e in device]) / 1000.0
    lines = [
        str(trace_path),
        "",
        f"  profiled steps        {n}",
        f"  mean step             {step_ms:8.1f} ms",
        f"  GPU busy              {busy_ms / n:8.1f} ms/step   {busy_ms / window_ms * 100:5.1f}%",
        f"  GPU idle              {(window_ms - busy_ms) / n:8.1f} ms/step   "
        f"{(window_ms - busy_ms) / window_ms * 100:5.1f}%   <- host could not keep the device fed",
        "",
    ]
    for cat, title in (("user_annotation", "host wall clock"), ("gpu_user_annotation", "device time")):
        totals: dict[str, float] = defaultdict(float)
        for e in cats.get(cat, []):
            if not str(e["name"]).startswith("ProfilerStep"):
                totals[str(e["name"])] += e["dur"] / 1000.0
        if not totals:
            continue
        lines += [f"  --- annotated regions, {title} ---", f"  {'region':<34}{'ms/step':>9}{'% step':>9}"]
        for name, total in sorted(totals.items(), key=lambda kv: -kv[1])[:12]:
            lines.append(f"  {name[:33]:<34}{total / n:>9.1f}{total / n / step_ms * 100:>8.1f}%")
        lines.append("")
    syncs = [e for e in cats.get("cuda_runtime", []) if "Synchronize" in str(e["name"])]
    if syncs:
        blocked = sum(e["dur"] for e in syncs) / 1000.0
        lines += [
            f"  host blocked in cudaStreamSynchronize & co: {blocked / n:.1f} ms/step over "
            f"{len(syncs) / n:.0f} calls/step",
            "",
        ]
    per_kernel: dict[str, list[float]] = defaultdict(lambda: [0.0, 0.0])
    for e in device:
        entry = per_kernel[str(e["name"])]
        entry[0] += e["dur"] / 1000.0
        entry[1] += 1
    lines += ["  --- slowest kernels ---", f"  {'kernel':<62}{'ms/step':>9}{'% step':>9}"]
    for name, (total, _) in sorted(per_kernel.items(), key=lambda kv: -kv[1][0])[:12]:
        lines.append(f"  {name[:61]:<62}{total / n:>9.2f}{total / n / step_ms * 100:>8.1f}%")
    lines += ["", "  Open the trace at https://ui.perfetto.dev for the full timeline:", f"    {trace_path}"]
    return "\n".join(lines)


def main() -> None:
    parser = argparse.ArgumentParser(
        prog="python -m mia_train_b200.engine.profiler", description="Summarise a run's profiler trace."
    )
    parser.add_argument("run", type=Path, help="a run directory, its profile/ directory, or a trace file")
    print(summarize(find_trace(parser.parse_args().run)))


if __name__ == "__main__":
    main()
