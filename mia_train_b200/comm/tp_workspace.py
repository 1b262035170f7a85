"""Peer-memory workspace of the fused tensor-parallel kernels (`csrc/tp_gemm.cu`).

One CUDA-IPC allocation per rank of the TP group, mapped into every peer:

    [ flags | gather area, parity 0 | parity 1 | receive slots, parity 0 | parity 1 ]

* flags: the per-block ready flags the peers write, local counters, and the device epochs that
  select the buffer parity of each launch (so a captured CUDA graph stays correct on replay);
* gather area: one (rows per rank, K) bf16 slot per source rank, into which every peer pushes its
  rows of an all-gathered operand;
* receive slots: one (rows per rank, N) bf16 slot per source rank, written by every peer's
  GEMM epilogue and added into this rank's accumulators.

Sizes are fixed at construction (`max_rows` rows per rank, at most `max_k` gathered columns and
`max_n` reduced columns); the kernels refuse larger problems. Construction is collective.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from ..ops._native import native
from .ipc import IpcBuffers


def _round256(n: int) -> int:
    return (n + 255) // 256 * 256


class TpWorkspace:
    def __init__(
        self,
        group: Any,
        device: torch.device,
        max_rows: int,
        max_k: int,
        max_n: int,
        timeout_ms: float = 10_000.0,
    ) -> None:
        self.group = group
        self.device = device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_rows, self.max_k, self.max_n = int(max_rows), int(max_k), int(max_n)
        self.timeout_ms = float(timeout_ms)
        self.flag_bytes = _round256(int(native().tp_flag_bytes()))
        self.gather_parity_bytes = _round256(self.world * self.max_rows * self.max_k * 2)
        self.recv_parity_bytes = _round256(self.world * self.max_rows * self.max_n * 2)
        total = self.flag_bytes + 2 * self.gather_parity_bytes + 2 * self.recv_parity_bytes
        self._ipc = IpcBuffers(group, device)
        self.local, peers = self._ipc.allocate(total, torch.uint8)
        self.flag_peers = [int(p) for p in peers]
        self.gather_peers = [p + self.flag_bytes for p in self.flag_peers]
        self.recv_peers = [p + self.flag_bytes + 2 * self.gather_parity_bytes for p in self.flag_peers]
        self.nbytes = total
        # B operand of the reduce-scatter kernel's identity MMA (adds received partials in TMEM)
        self.ident = torch.eye(128, dtype=torch.bfloat16, device=device)

    def release(self) -> None:
        self._ipc.release()

    # -- the two fused launches ------------------------------------------------------------------
    def ag_gemm(self, a_local, b, out, a_full, bias, aux, aux_out, b_kmajor: bool, act: int) -> None:
        if a_local.shape[0] > self.max_rows or a_local.shape[1] > self.max_k:
            raise ValueError(
                f"all-gather GEMM operand ({a_local.shape[0]} rows x {a_local.shape[1]}) exceeds the TP workspace "
                f"({self.max_rows} rows x {self.max_k})"
            )
        native().tp_ag_gemm(a_local, b, out, a_full, bias, aux, aux_out, b_kmajor, act, self.flag_peers,
                            self.gather_peers, self.gather_parity_bytes, self.rank, self.timeout_ms)

    def gemm_rs(self, a, b, out, bias, gamma, residual, pre_out, b_kmajor: bool) -> None:
        rows = a.shape[0] // self.world
        n = b.shape[0] if b_kmajor else b.shape[1]
        if rows > self.max_rows or n > self.max_n:
            raise ValueError(
                f"GEMM reduce-scatter output ({rows} rows x {n}) exceeds the TP workspace "
                f"({self.max_rows} rows x {self.max_n})"
            )
        native().tp_gemm_rs(a, b, out, bias, gamma, residual, pre_out, b_kmajor, self.flag_peers, self.recv_peers,
                            self.recv_parity_bytes, self.rank, self.timeout_ms, self.ident)
