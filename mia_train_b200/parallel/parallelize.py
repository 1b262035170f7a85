"""Apply tensor parallelism, then FSDP2 sharding or DDP replication, to a model or algorithm.

Same order and entry-point handling as the reference's `src/distributed/parallelize.py:16-103`
(TP first, then `fully_shard` of the model with its extra forward methods registered, then of the
algorithm with `validation_step` registered; `replicate` of the whole algorithm when only
`dp_replicate > 1`). Two differences, both selectable in `[parallelism]`:

* `fsdp_unit = "block"` (default) first shards every block the model and algorithm declare through
  `checkpointable_modules()` as its own unit, so parameters are gathered one block ahead of use and
  freed after it, instead of the whole encoder staying resident for the entire forward.
* `param_dtype = "bf16"` (default) gathers parameters in bf16 through `MixedPrecisionPolicy`, with
  fp32 gradient reduction. Under bf16 autocast the matmuls consumed bf16 weights anyway.
"""

from __future__ import annotations

import torch
import torch.nn as nn
from torch.distributed.device_mesh import DeviceMesh

try:
    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard, register_fsdp_forward_method
except ImportError:  # pragma: no cover - older torch
    from torch.distributed._composable.fsdp import (  # type: ignore[no-redef]
        MixedPrecisionPolicy,
        fully_shard,
        register_fsdp_forward_method,
    )
from torch.distributed._composable.replicate import replicate
from torch.distributed.tensor.parallel import parallelize_module

from ..algorithms.base import BaseAlgorithm
from ..models.base import BaseModel
from .parallel_dims import ParallelDims
from .tensor_parallel import BlockTensorParallelPlan, apply_tensor_parallel


def _apply_tensor_parallel(model: nn.Module, mesh: DeviceMesh, dims: ParallelDims) -> None:
    if not dims.tp_enabled:
        return
    adapted = [name for name, m in model.named_modules() if hasattr(m, "lora_a")]
    if adapted:
        # the tensor-parallel block paths read the base weights and would skip the adapters
        raise ValueError(
            f"[lora] adapters ({adapted[0]}, ... {len(adapted)} layers) cannot be combined with tensor "
            f"parallelism (tp = {dims.tp}): train the adapters with data parallelism (dp_shard / dp_replicate)"
        )
    dropping = [name for name, m in model.named_modules() if getattr(m, "sample_drop_ratio", 0.0) > 0.0]
    if dropping and dims.tp_comm != "allreduce":
        # stochastic depth trains a random subset of samples per block; the sequence-parallel
        # blocks hold token rows of every sample and have no subset path
        raise ValueError(
            f"drop_path ({dropping[0]}, ... {len(dropping)} blocks) cannot be combined with sequence-parallel "
            f"tensor parallelism (tp = {dims.tp}, tp_comm = {dims.tp_comm!r}): set [model] drop_path_rate = 0, "
            "use tp_comm = \"allreduce\", or train with data parallelism"
        )
    plan = model.tensor_parallel_plan() if isinstance(model, BaseModel) else None
    if plan is None:
        raise ValueError(
            f"{type(model).__name__} does not define a tensor_parallel_plan(), but tp={dims.tp} was requested"
        )
    if isinstance(plan, BlockTensorParallelPlan):
        group = mesh["tp"].get_group()
        apply_tensor_parallel(plan, group)
        enable = getattr(model, "enable_sequence_parallel", None)
        if dims.tp_comm != "allreduce" and enable is not None:
            from ..ops.tp import TpComm
            from .sequence_parallel import SequenceParallel

            enable(SequenceParallel(TpComm(group, dims.tp_comm)))
        return
    parallelize_module(model, mesh["tp"], plan)
    prepare = getattr(model, "after_tensor_parallel", None)
    if prepare is not None:
        prepare(mesh["tp"])


def _dp_mesh(mesh: DeviceMesh, dims: ParallelDims) -> DeviceMesh | None:
    if dims.hsdp_enabled:
        return mesh["dp_replicate", "dp_shard"]
    if dims.dp_shard > 1:
        return mesh["dp_shard"]
    return None


def _mp_policy(dims: ParallelDims) -> MixedPrecisionPolicy:
    if dims.param_dtype == "bf16":
        return MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
    return MixedPrecisionPolicy()


def _shard(module: nn.Module, mesh: DeviceMesh, dims: ParallelDims, reshard: bool = True) -> bool:
    dp_mesh = _dp_mesh(mesh, dims)
    if dp_mesh is None:
        return False
    fully_shard(module, mesh=dp_mesh, mp_policy=_mp_policy(dims), reshard_after_forward=reshard)
    return True


def _entry_points(model: nn.Module) -> tuple[str, ...]:
    return model.extra_forward_methods() if isinstance(model, BaseModel) else ()


def _shard_unit(module: nn.Module, mesh: DeviceMesh, dims: ParallelDims) -> None:
    """Shard `module` as one FSDP unit, registering a model's extra entry points. A container without
    a forward of its own (a `ModuleDict` such as a teacher's backbone and heads) cannot be a unit:
    each of its children with parameters is sharded instead."""
    if type(module).forward is nn.Module.forward:
        for child in module.children():
            if any(True for _ in child.parameters()):
                _shard_unit(child, mesh, dims)
        return
    if _shard(module, mesh, dims):
        for name in _entry_points(module):
            register_fsdp_forward_method(module, name)


def _shard_blocks(root: nn.Module, mesh: DeviceMesh, dims: ParallelDims) -> int:
    """Shard every declared block (model's and algorithm's) as its own FSDP2 unit."""
    if dims.fsdp_unit != "block" or _dp_mesh(mesh, dims) is None:
        return 0
    seen: set[int] = set()
    count = 0
    for module in root.modules():
        if not isinstance(module, (BaseModel, BaseAlgorithm)):
            continue
        for block in module.checkpointable_modules():
            if id(block) in seen or not any(True for _ in block.parameters()):
                continue
            seen.add(id(block))
            _shard(block, mesh, dims)
            count += 1
    return count


def parallelize_model(model: nn.Module, mesh: DeviceMesh, dims: ParallelDims) -> nn.Module:
    """For a model used only through its own methods (no algorithm around it)."""
    _apply_tensor_parallel(model, mesh, dims)
    entries = _entry_points(model)
    _shard_blocks(model, mesh, dims)
    if _shard(model, mesh, dims):
        for name in entries:
            register_fsdp_forward_method(model, name)
    elif dims.dp_replicate > 1:
        if entries:
            raise ValueError(
                f"{type(model).__name__} is also used through {entries} rather than only forward(); "
                "`replicate` all-reduces gradients from forward hooks and would skip those calls. "
                "Replicate the owning algorithm instead (parallelize_algorithm)."
            )
        replicate(model, device_mesh=mesh["dp_replicate"])
    return model


def parallelize_algorithm(algorithm: BaseAlgorithm, mesh: DeviceMesh, dims: ParallelDims) -> BaseAlgorithm:
    """Parallelize a strategy and its model; the algorithm is the outer FSDP unit."""
    _apply_tensor_parallel(algorithm.model, mesh, dims)
    # models that must share the main model's tensor-parallel layout (a teacher updated from it)
    for extra_model in getattr(algorithm, "extra_tensor_parallel_models", lambda: ())():
        _apply_tensor_parallel(extra_model, mesh, dims)
    _shard_blocks(algorithm, mesh, dims)
    if _shard(algorithm.model, mesh, dims):
        for name in _entry_points(algorithm.model):
            register_fsdp_forward_method(algorithm.model, name)
    extra = getattr(algorithm, "extra_sharded_modules", None)
    if extra is not None:
        for module in extra():
            _shard_unit(module, mesh, dims)
    if _shard(algorithm, mesh, dims):
        register_fsdp_forward_method(algorithm, "validation_step")
    elif dims.dp_replicate > 1:
        replicate(algorithm, device_mesh=mesh["dp_replicate"])
    return algorithm


def refresh_fsdp_grad_dtypes(root: nn.Module) -> int:
    """Re-derive every FSDP2 unit's gradient dtypes after `requires_grad` changed.

    FSDP2 takes a unit's reduce and original dtypes from the parameters that require grad when it
    first runs; a unit whose parameters were all frozen then (a backbone frozen for the first
    steps) keeps none, so once unfrozen it reduces gradients in the bf16 compute dtype and assigns
    them to fp32 parameters, which autograd refuses. Returns the number of units refreshed."""
    count = 0
    for module in root.modules():
        get_state = getattr(module, "_get_fsdp_state", None)
        group = getattr(get_state(), "_fsdp_param_group", None) if get_state is not None else None
        if group is not None:
            group._init_mp_dtypes()
            count += 1
    return count
