"""The `[parallelism]` section: a 3-D mesh `(dp_replicate, dp_shard, tp)`.

Same semantics as the reference's `src/distributed/parallel_dims.py:9-60`: the product must equal
the world size, tensor-parallel peers read the same batch, and
`dp_rank = replicate_rank * dp_shard + shard_rank`.

New keys (defaults keep reference configs valid):
* `fsdp_unit` -- `"block"` shards every transformer block as its own FSDP2 unit (prefetch and
  resharding per block); `"model"` reproduces the reference's two coarse units.
* `param_dtype` -- dtype FSDP2 all-gathers parameters in (`"bf16"` halves the traffic of the
  reference's fp32 gather; `"fp32"` reproduces it). Gradients are always reduced in fp32.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh

FSDP_UNITS = ("block", "model")
PARAM_DTYPES = ("bf16", "fp32")


@dataclass(frozen=True)
class ParallelDims:
    dp_replicate: int = 1
    dp_shard: int = 1
    tp: int = 1
    fsdp_unit: str = "block"
    param_dtype: str = "bf16"

    def __post_init__(self) -> None:
        if self.dp_replicate < 1 or self.dp_shard < 1 or self.tp < 1:
            raise ValueError(f"dp_replicate, dp_shard, and tp must all be >= 1, got {self}")
        if self.fsdp_unit not in FSDP_UNITS:
            raise ValueError(f"fsdp_unit must be one of {FSDP_UNITS}, got {self.fsdp_unit!r}")
        if self.param_dtype not in PARAM_DTYPES:
            raise ValueError(f"param_dtype must be one of {PARAM_DTYPES}, got {self.param_dtype!r}")

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
                f"process group world_size={actual} does not match dp_replicate({self.dp_replicate}) "
                f"* dp_shard({self.dp_shard}) * tp({self.tp}) = {self.world_size}"
            )
        return init_device_mesh(
            device_type,
            (self.dp_replicate, self.dp_shard, self.tp),
            mesh_dim_names=("dp_replicate", "dp_shard", "tp"),
        )
