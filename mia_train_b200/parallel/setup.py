"""Process-group setup from torchrun's environment (reference `src/distributed/setup.py:9-33`).

NCCL when CUDA is present, Gloo otherwise. The process group gets a bounded timeout
(`MIA_PG_TIMEOUT_S`, default 600 s) so that ranks waiting on a dead peer end with an error instead of
hanging for NCCL's default of ten minutes or more.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def default_backend() -> str:
    return "nccl" if torch.cuda.is_available() else "gloo"


def device_type() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"


def init_distributed(backend: str | None = None, timeout_s: float | None = None) -> tuple[int, int, int]:
    """Initialise the default process group; returns (rank, world_size, local_rank)."""
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    if not dist.is_initialized():
        if "RANK" not in os.environ:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29512")
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
        timeout = timeout_s if timeout_s is not None else float(os.environ.get("MIA_PG_TIMEOUT_S", "600"))
        kwargs = {"timeout": datetime.timedelta(seconds=timeout)}
        if torch.cuda.is_available() and (backend or default_backend()) == "nccl":
            kwargs["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(backend=backend or default_backend(), **kwargs)
    return dist.get_rank(), dist.get_world_size(), local_rank


def destroy_distributed() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
