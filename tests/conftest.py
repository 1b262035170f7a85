"""Shared fixtures: the `gpu` marker, a CPU Gloo multi-process harness, and tiny configs."""

from __future__ import annotations

import os
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the native extension")
    config.addinivalue_line("markers", "cpu_dist: multi-process CPU test over the Gloo backend")
    config.addinivalue_line("markers", "slow: long-running test")


def _worker(rank: int, world_size: int, init_file: str, fn, args, queue) -> None:  # noqa: ANN001
    import torch.distributed as dist

    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world_size)
    os.environ["LOCAL_RANK"] = str(rank)
    try:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world_size)
        torch.manual_seed(0)
        result = fn(rank, world_size, *args)
        queue.put((rank, "ok", result))
    except BaseException as error:  # noqa: BLE001
        queue.put((rank, "error", f"{type(error).__name__}: {error}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.fixture
def run_distributed(tmp_path):
    """run_distributed(fn, world_size, *args) -> {rank: result}; fn(rank, world_size, *args)."""

    calls = [0]

    def launch(fn, world_size: int = 2, *args, timeout: float = 240.0):
        ctx = mp.get_context("spawn")
        queue = ctx.Queue()
        calls[0] += 1  # a fresh rendezvous file per launch: a used one holds the last group's state
        init_file = str(tmp_path / f"pg_init_{os.getpid()}_{calls[0]}")
        procs = [
            ctx.Process(target=_worker, args=(r, world_size, init_file, fn, args, queue), daemon=True)
            for r in range(world_size)
        ]
        for p in procs:
            p.start()
        results, errors = {}, []
        try:
            for _ in range(world_size):
                rank, status, payload = queue.get(timeout=timeout)
                if status == "ok":
                    results[rank] = payload
                else:
                    errors.append(f"rank {rank}: {payload}")
        finally:
            for p in procs:
                p.join(timeout=10)
                if p.is_alive():
                    p.kill()
        if errors:
            raise AssertionError("\n".join(errors))
        return results

    return launch


@pytest.fixture
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    return torch.device("cuda", 0)
