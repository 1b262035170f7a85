"""CUDA-IPC peer memory: buffers every rank of a process group can read and write over NVLink.

Each rank allocates with `cudaMalloc` and exports a CUDA IPC handle (`_C.ipc_export`); the
handles are exchanged over the process group and opened on every peer (`_C.ipc_open`), which gives
every rank a device pointer to every peer's copy. Kernels move data with plain peer loads and
stores (`csrc/comm.cu`) or with TMA stores and bulk copies into the peers' buffers
(`csrc/tp_gemm.cu`). Allocation is collective: every rank of the group must
call `allocate` with the same sizes in the same order.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from ..ops._native import native


class IpcBuffers:
    """Device buffers allocated with cudaMalloc and mapped into every peer through CUDA IPC."""

    def __init__(self, group: Any, device: torch.device) -> None:
        self.group = group
        self.device = device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._owned: list[tuple[list[int], int]] = []

    def allocate(self, numel: int, dtype: torch.dtype) -> tuple[torch.Tensor, list[int]]:
        """(local tensor, [device pointer of every rank's copy]) -- a collective call."""
        elem = torch.empty((), dtype=dtype).element_size()
        nbytes = max(numel * elem, 256)
        local, handle, addr = native().ipc_export(nbytes, self.device.index)
        handles = [torch.empty_like(handle) for _ in range(self.world)]
        gathered = all_gather_cpu(handle, self.group)
        for h, g in zip(handles, gathered, strict=True):
            h.copy_(g)
        peers = native().ipc_open(torch.stack(handles), self.rank, int(addr[0]), self.device.index)
        self._owned.append((peers, int(addr[0])))
        return local.view(dtype)[:numel], peers

    def release(self) -> None:
        if not self._owned:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every peer stopped using our memory
        for peers, _ in self._owned:
            native().ipc_close(peers, self.rank, self.device.index)
        dist.barrier(group=self.group)  # every peer closed its mapping of ours
        for _, addr in self._owned:
            native().ipc_free(addr, self.device.index)
        self._owned = []


def all_gather_cpu(t: torch.Tensor, group: Any) -> list[torch.Tensor]:
    """All-gather a small CPU byte tensor through whatever backend the group uses."""
    if dist.get_backend(group) == "nccl":
        dev = torch.device("cuda", torch.cuda.current_device())
        src = t.to(dev)
        out = [torch.empty_like(src) for _ in range(dist.get_world_size(group))]
        dist.all_gather(out, src, group=group)
        return [o.cpu() for o in out]
    out = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, t, group=group)
    return out
