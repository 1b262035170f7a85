"""Windowed DINOv3 ViT-L SimMIM at 256^3 / patch 8 under sequence-parallel TP (the `bench.py --config
windowed_tp` workload).

Workload: `dinov3_vit3d` dim 1024 / depth 24 / 16 heads / GELU MLP 4096, patch 8^3 on single-channel
256^3 volumes (32^3 = 32768 patch tokens + a class token), 8^3-token attention windows with a
global block every 6th block, 3D RoPE; `simmim` with mask ratio 0.6 (mask-token substitution, L1 on
masked voxels); bf16 autocast; activation checkpointing of every block; per-replica batch 1; AdamW
(lr 1.5e-4, betas 0.9 / 0.95, wd 0.05), grad clip 1.0. Data: uint8 volumes of blurred Gaussian
noise plus Poisson(50) ellipsoids, z-scored per volume on the device inside the step.

Layout on N GPUs: TP = min(4, N) ranks share one sample (sequence-parallel blocks), and
N / TP data-parallel replicas each take one sample, so the global batch is N / TP.

* native arm: this framework. `tp_comm = "fused"` runs every block GEMM as a fused all-gather ->
  GEMM or GEMM -> reduce-scatter kernel over NVLink peer memory; `"collective"` is the same
  layout on NCCL collectives (the framework's own NCCL baseline). Data-parallel gradients are one
  NCCL all-reduce of the flat fp32 gradient buffer; the per-token-shard norm gradients are summed
  over the TP group; the clip norm counts sharded parameters over the TP group and replicated ones
  once; AdamW is the fused native optimizer.
* reference arm: the unmodified reference package (baseline/_ref) through its own Trainer, model
  and algorithm objects -- it has no TP plan and no windowed attention, so it runs the same model
  with global attention on FSDP2 dp_shard = N with activation checkpointing, per-rank batch 1.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path
from typing import Any, Callable

import torch
import torch.distributed as dist

MODEL = dict(img_size=256, patch_size=8, embed_dim=1024, depth=24, num_heads=16, ffn_ratio=4.0)
WINDOW = dict(window_size=8, global_every=6)
MASK_RATIO = 0.6
SIDE = 256
METRIC = ("samples/sec (windowed dinov3_vit3d ViT-L SimMIM, 256^3, patch 8, bf16), whole box, "
          "device-timed max over ranks")
DATA = "synthetic (uint8 blurred-noise + ellipsoid 256^3 volumes, z-scored on device; random-init weights)"
SEQ_LEN = 32769  # 32768 patch tokens + class token


def describe(n_gpus: int) -> dict:
    tp = min(4, n_gpus)
    return {
        "model": "dinov3_vit3d ViT-L (1024/24/16, MLP 4096), windows 8^3 + global every 6th block, simmim mask 0.6",
        "img": "256^3 / patch 8 (32768 tokens + class token)",
        "tp": tp,
        "dp": n_gpus // tp,
        "activation_checkpointing": True,
    }


def make_volumes(n: int, seed: int, side: int = SIDE) -> torch.Tensor:
    """n uint8 volumes (n, 1, 1, side, side, side): blurred noise + ellipsoid blobs."""
    from ..data.synthetic import blobs_volume

    vols = []
    for i in range(n):
        g = torch.Generator().manual_seed(seed * 1000 + i)
        v = blobs_volume((side,) * 3, 3.0, 50.0, (2.0, 8.0), g)
        vols.append(((v - v.min()) / (v.max() - v.min()).clamp_min(1e-6) * 255).round().to(torch.uint8))
    return torch.stack(vols)[:, None, None].contiguous()


def _groups(world: int, tp: int) -> tuple[Any, Any, int]:
    """(TP group, DP group, dp rank) for consecutive-rank TP groups."""
    rank = dist.get_rank()
    tp_group = dp_group = None
    for start in range(0, world, tp):
        ranks = list(range(start, start + tp))
        g = dist.new_group(ranks)
        if rank in ranks:
            tp_group = g
    for j in range(tp):
        ranks = list(range(j, world, tp))
        g = dist.new_group(ranks)
        if rank in ranks:
            dp_group = g
    return tp_group, dp_group, rank // tp


def native_arm(args: Any, rank: int, world: int, local: int, clock_sampler: Callable, timed: Callable,
               kernel_table: Callable | None = None) -> dict:
    from .. import components  # noqa: F401
    from ..algorithms.simmim import SimMIM
    from ..engine.activation_checkpoint import apply_activation_checkpointing
    from ..engine.config import TrainerConfig
    from ..engine.graph_step import FlatParameters
    from ..engine.optimizer import build_optimizer
    from ..models.dinov3_vit3d import DinoVisionTransformer3D
    from ..ops import _native
    from ..ops.data import zscore_u8
    from ..ops.optim import clip_coefficient, grad_sumsq
    from ..ops.tp import TpComm
    from ..parallel.sequence_parallel import SequenceParallel, partial_params, sync_partial_grads
    from ..parallel.tensor_parallel import apply_tensor_parallel, is_tensor_parallel

    _native.native()
    dev = torch.device("cuda", local)
    tp = min(4, world)
    tp_group, dp_group, dp_rank = _groups(world, tp) if world > 1 else (None, None, 0)
    torch.manual_seed(0)
    model = DinoVisionTransformer3D(**MODEL, **WINDOW)
    alg = SimMIM(model, input_axes="lcxyz", mask_ratio=MASK_RATIO).to(dev)
    if world > 1:
        for p in alg.parameters():
            dist.broadcast(p.data, 0)
    comm = None
    if tp > 1:
        apply_tensor_parallel(model.tensor_parallel_plan(), tp_group)
        comm = TpComm(tp_group, args.tp_comm)
        model.enable_sequence_parallel(SequenceParallel(comm))
    apply_activation_checkpointing(alg)
    flat = FlatParameters(alg)
    tcfg = TrainerConfig(max_steps=args.warmup + 2 * args.steps + 8, batch_size=1, lr=1.5e-4, weight_decay=0.05,
                         beta1=0.9, beta2=0.95, warmup_steps=2, precision="bf16", grad_clip_norm=1.0,
                         fused_optimizer="on")
    opt = build_optimizer(alg, tcfg)
    # parameters that differ between TP ranks: sharded weights and the biases of qkv / column layers
    sharded = [p for m in alg.modules() if is_tensor_parallel(m) for name, p in m.named_parameters(recurse=False)
               if p.requires_grad and (name == "weight" or m._tp_mode != "row")]
    sharded_ids = {id(p) for p in sharded}
    replicated = [p for p in alg.parameters() if p.requires_grad and id(p) not in sharded_ids]
    # every TP rank of a replica must draw the same SimMIM mask: one CUDA RNG stream per replica
    torch.cuda.manual_seed(1234 + dp_rank)

    pool_cpu = make_volumes(2, seed=dp_rank + 1)
    pool_dev = pool_cpu.to(dev)
    pool_pinned = pool_cpu.pin_memory()

    def step(u8: torch.Tensor) -> torch.Tensor:
        flat.grad.zero_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = alg({"img": zscore_u8(u8, torch.bfloat16)})
        out["loss"].backward()
        alg.zero_grad(set_to_none=True)  # every gradient is in the flat buffer (main_grad) now
        if comm is not None:
            sync_partial_grads(alg)
        if dp_group is not None and dist.get_world_size(dp_group) > 1:
            dist.all_reduce(flat.grad, group=dp_group)
        sq_sh = grad_sumsq([p.main_grad for p in sharded]) if sharded else torch.zeros((), device=dev)
        if tp_group is not None:
            dist.all_reduce(sq_sh, group=tp_group)
        sq = sq_sh + grad_sumsq([p.main_grad for p in replicated])
        dp = dist.get_world_size(dp_group) if dp_group is not None else 1
        opt.grad_scale = clip_coefficient(sq.sqrt() / dp, 1.0) / dp
        opt.step()
        return out["loss"]

    for i in range(args.warmup):
        step(pool_dev[i % 2:i % 2 + 1])
    torch.cuda.synchronize()
    if getattr(args, "profile_kernels", 0) and kernel_table is not None:
        table = kernel_table(lambda: step(pool_dev[0:1]) and None, args.profile_kernels)
        if rank == 0:
            print(table, flush=True)
    ms, loss, clocks = timed(lambda i: step(pool_dev[i % 2:i % 2 + 1]), args.steps, clock_sampler)
    e2e = None
    if not args.no_e2e:
        def e2e_step(i: int) -> torch.Tensor:
            u8 = pool_pinned[i % 2:i % 2 + 1].to(dev, non_blocking=True)
            loss_i = step(u8)
            _ = loss_i.item()
            return loss_i

        e2e_ms, _, _ = timed(e2e_step, args.steps, None)
        e2e = {"ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": SIDE**3, "d2h_bytes_per_step": 4,
               "api": "mia_train_b200 SimMIM + sequence-parallel dinov3_vit3d (eager step)"}
    errors = int(_native.native().check_errors(local))
    n_partial = len(partial_params(alg))
    flops = _step_flops(model, alg, tp)
    if comm is not None:
        comm.release()
    return {"ms": ms, "loss": float(loss), "clocks": clocks, "e2e": e2e, "errors": errors, "flops": flops,
            "global_batch": world // tp, "lib": _native.loaded_library_path(), "partial_params": n_partial,
            "parallelism": f"tp{tp} x dp{world // tp} ({args.tp_comm if tp > 1 else 'no TP'}), activation checkpointing"}


def _step_flops(model: Any, alg: Any, tp: int) -> float:
    """Per-rank FLOPs of one step: forward, recomputed forward (checkpointing) and backward (2x)."""
    fwd = model.flops((1, SIDE, SIDE, SIDE)) + 2 * model.num_patches * model.embed_dim * math.prod(alg.patch_size)
    return 4.0 * fwd / tp


def reference_arm(args: Any, rank: int, world: int, local: int, clock_sampler: Callable, timed: Callable,
                  repo: Path) -> dict:
    ref_root = repo / "baseline" / "_ref"
    if not (ref_root / "engine" / "trainer.py").is_file():
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    from algorithms.simmim import SimMIM as RefSimMIM  # type: ignore
    from data.base import BaseDataset as RefBase  # type: ignore
    from distributed.parallel_dims import ParallelDims  # type: ignore
    from engine.config import TrainerConfig as RefTrainerConfig  # type: ignore
    from engine.trainer import Trainer as RefTrainer  # type: ignore
    from models.dinov3_vit3d import DinoVisionTransformer3D as RefDino  # type: ignore

    dev = torch.device("cuda", local)
    pool = make_volumes(2, seed=rank + 1)

    def zscore(u8: torch.Tensor) -> torch.Tensor:
        v = u8.float()
        dims = tuple(range(1, v.dim()))
        return (v - v.mean(dim=dims, keepdim=True)) / v.std(dim=dims, keepdim=True).clamp_min(1e-6)

    vols = zscore(pool)

    class SyntheticVolumes(RefBase):
        def build_dataset(self):
            return torch.utils.data.TensorDataset(vols)

        @property
        def sample_axes(self):
            return "lcxyz"

    torch.manual_seed(0)
    model = RefDino(**MODEL)
    ds = SyntheticVolumes()
    alg = RefSimMIM(model, ds, mask_ratio=MASK_RATIO)
    tcfg = RefTrainerConfig(max_steps=args.warmup + 2 * args.steps + 8, batch_size=1, lr=1.5e-4, weight_decay=0.05,
                            beta1=0.9, beta2=0.95, warmup_steps=2, precision="bf16", grad_clip_norm=1.0,
                            measure_mfu=False, activation_checkpointing=True)
    dims = ParallelDims(dp_shard=world) if world > 1 else ParallelDims()
    mesh = dims.build_mesh("cuda") if world > 1 else None
    trainer = RefTrainer(alg, ds, tcfg, Path("/tmp") / f"ref_c4_{os.getpid()}", dims=dims, mesh=mesh, device=dev)

    def step(u8: torch.Tensor) -> torch.Tensor:
        batch = {"img": zscore(u8)}
        with trainer._autocast():
            metrics = trainer.algorithm(batch)
        metrics["loss"].backward()
        torch.nn.utils.clip_grad_norm_(trainer.algorithm.parameters(), tcfg.grad_clip_norm)
        trainer.optimizer.step()
        trainer.scheduler.step()
        trainer.optimizer.zero_grad(set_to_none=True)
        return metrics["loss"]

    pool_dev = pool.to(dev)
    pool_pinned = pool.pin_memory()
    for i in range(args.warmup):
        step(pool_dev[i % 2:i % 2 + 1])
    torch.cuda.synchronize()
    ms, loss, clocks = timed(lambda i: step(pool_dev[i % 2:i % 2 + 1]), args.steps, clock_sampler)
    e2e = None
    if not args.no_e2e:
        def e2e_step(i: int) -> torch.Tensor:
            loss_i = step(pool_pinned[i % 2:i % 2 + 1].to(dev, non_blocking=True))
            _ = loss_i.item()
            return loss_i

        e2e_ms, _, _ = timed(e2e_step, args.steps, None)
        e2e = {"ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": SIDE**3, "d2h_bytes_per_step": 4,
               "api": "reference Trainer objects, eager step"}
    # the reference model is all-global: count its forward with the same analytic formula
    from ..models.dinov3_vit3d import DinoVisionTransformer3D

    with torch.device("meta"):
        meta = DinoVisionTransformer3D(**MODEL)
    fwd = meta.flops((1, SIDE, SIDE, SIDE)) + 2 * meta.num_patches * meta.embed_dim * 8**3
    return {"ms": ms, "loss": float(loss), "clocks": clocks, "e2e": e2e, "flops": 4.0 * fwd, "global_batch": world,
            "parallelism": f"FSDP2 dp_shard={world}, global attention, activation checkpointing"}
