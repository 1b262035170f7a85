"""The `[parallelism]` section: a 3-D mesh `(dp_replicate, dp_shard, tp)`.

Same semantics as the reference's `src/distributed/parallel_dims.py:9-60`: the product must equal
the world size, tensor-parallel peers read the same batch, and
`dp_rank = replicate_rank * dp_shard + shard_rank`.

New keys (defaults keep reference configs valid):
* `fsdp_unit` -- `"block"` shards every transformer block as its own FSDP2 unit (prefetch and
  resharding per block); `"model"` reproduces the reference's two coarse units.
* `param_dtype` -- dtype FSDP2 all-gathers parameters in (`"bf16"` halves the traffic of the
  reference's fp32 gather; `"fp32"` reproduces it). Gradients are always reduced in fp32.
* `tp_comm` -- how tensor-parallel blocks communicate: `"fused"` (sequence-parallel, the
  all-gather -> GEMM and GEMM -> reduce-scatter kernels over NVLink peer memory; on CPU the same
  layout on collectives), `"collective"` (sequence-parallel on NCCL / Gloo collectives) or
  `"allreduce"` (replicated activations, one all-reduce per row-parallel layer).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh

FSDP_UNITS = ("block", "model")
PARAM_DTYPES = ("bf16", "fp32")
TP_COMMS = ("fused", "collective", "allreduce")


@dataclass(frozen=True)
class ParallelDims:
    dp_replicate: int = 1
    dp_shard: int = 1
    tp: int = 1
    fsdp_unit: str = "block"
    param_dtype: str = "bf16"
    tp_comm: str = "fused"

    def __post_init__(self) -> None:
        sizes = {"dp_replicate": self.dp_replicate, "dp_shard": self.dp_shard, "tp": self.tp}
        bad = [f"{k} = {v}" for k, v in sizes.items() if v < 1]
        if bad:
            raise ValueError(f"[parallelism]: every mesh dimension is a positive size ({', '.join(bad)})")
        if self.fsdp_unit not in FSDP_UNITS:
            raise ValueError(f"[parallelism]: fsdp_unit {self.fsdp_unit!r} is not one of {', '.join(FSDP_UNITS)}")
        if self.param_dtype not in PARAM_DTYPES:
            raise ValueError(f"[parallelism]: param_dtype {self.param_dtype!r} is not one of {', '.join(PARAM_DTYPES)}")
        if self.tp_comm not in TP_COMMS:
            raise ValueError(f"[parallelism]: tp_comm {self.tp_comm!r} is not one of {', '.join(TP_COMMS)}")

    @property
    def world_size(self) -> int:
        return self.dp_replicate * self.dp_shard * self.tp

    @property
    def dp_enabled(self) -> bool:
        return self.dp_replicate > 1 or self.dp_shard > 1

    @property
    def hsdp_enabled(self) -> bool:
        return self.dp_replicate > 1 and self.dp_shard > 1

    @property
    def tp_enabled(self) -> bool:
        return self.tp > 1

    @property
    def dp_world_size(self) -> int:
        return self.dp_replicate * self.dp_shard

    def dp_rank(self, mesh: DeviceMesh) -> int:
        rep = mesh.get_local_rank("dp_replicate") if self.dp_replicate > 1 else 0
        shard = mesh.get_local_rank("dp_shard") if self.dp_shard > 1 else 0
        return rep * self.dp_shard + shard

    def build_mesh(self, device_type: str) -> DeviceMesh:
        actual = dist.get_world_size()
        if actual != self.world_size:
            raise ValueError(
                f"[parallelism] describes a mesh of {self.world_size} ranks ({self.dp_replicate} replicas x "
                f"{self.dp_shard} shards x tp {self.tp}), but {actual} processes were launched"
            )
        return init_device_mesh(
            device_type,
            (self.dp_replicate, self.dp_shard, self.tp),
            mesh_dim_names=("dp_replicate", "dp_shard", "tp"),
        )
