"""Affinity segmentation with a ViT-L 3D encoder and a sub-pixel decoder at 128^3 / patch 8 under
sequence-parallel TP (the `bench.py --config affinity_tp` workload).

Workload: `dinov3_vit3d` dim 1024 / depth 24 / 16 heads / GELU MLP 4096, patch 8^3 on 128^3
volumes (16^3 = 4096 patch tokens + a class token), global attention, 3D RoPE; `affinity_seg` with
the `"subpixel"` decoder predicting 12 affinity channels (`offsets = "nisb12"`: 3 nearest-neighbour
plus 9 long-range offsets up to 9 voxels) trained with masked BCE; bf16 autocast; per-replica batch
4; AdamW (lr 1e-4, wd 0.05), grad clip 1.0. Data: uint32 instance labels made as 3-D Voronoi cells
from 300 uniform seeds with a 1-voxel boundary zeroed; raw input per-cell mean intensity U[0.3, 0.7],
membranes darkened by 0.4, Gaussian noise sigma 0.08, blurred with sigma 1 voxel, stored as bf16.
Connected components are not re-split inside the step (the training engine does that in the data
loader workers).

Layout on N GPUs: TP = min(2, N) ranks share a replica's 4 samples (sequence-parallel encoder
blocks; the decoder and loss run on the gathered tokens on every TP rank), N / TP replicas.

* native arm: this framework, `tp_comm = "fused"` (fused collective-GEMM kernels over NVLink) or
  `"collective"` (NCCL), the same gradient / clip / AdamW handling as the windowed-TP benchmark.
* reference arm: the unmodified reference (baseline/_ref) through its own Trainer, model and
  algorithm objects on FSDP2 dp_shard = N with per-rank batch 4; it has no tensor-parallel plan and
  only its 6-channel affinity layout (3 nearest-neighbour + 3 long-range at `long_range`).
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path
from typing import Any, Callable

import torch
import torch.distributed as dist

MODEL = dict(img_size=128, patch_size=8, embed_dim=1024, depth=24, num_heads=16, ffn_ratio=4.0)
SIDE = 128
METRIC = ("samples/sec (affinity_seg ViT-L 3D + sub-pixel decoder, 128^3, patch 8, 12 offsets, bf16), whole box, "
          "device-timed max over ranks")
DATA = ("synthetic (3-D Voronoi instance labels from 300 seeds, membrane-darkened noisy bf16 images; "
        "random-init weights)")
SEQ_LEN = 4097  # 4096 patch tokens + class token
BATCH = 4


def describe(n_gpus: int) -> dict:
    tp = min(2, n_gpus)
    return {
        "model": "dinov3_vit3d ViT-L (1024/24/16, MLP 4096) + affinity_seg sub-pixel decoder, 12 offsets",
        "img": "128^3 / patch 8 (4096 tokens + class token)",
        "tp": tp,
        "dp": n_gpus // tp,
        "per_replica_batch": BATCH,
    }


def make_samples(n: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(images (n, 1, 1, D, H, W) bf16, labels (n, 1, D, H, W) int32) of the Voronoi generator."""
    from ..data.synthetic import voronoi_volume

    imgs, labs = [], []
    for i in range(n):
        g = torch.Generator().manual_seed(seed * 1000 + i)
        img, lab = voronoi_volume((SIDE,) * 3, 300, 0.08, 1.0, g)
        imgs.append(img.to(torch.bfloat16))
        labs.append(lab.to(torch.int32))
    return torch.stack(imgs)[:, None, None].contiguous(), torch.stack(labs)[:, None].contiguous()


def native_arm(args: Any, rank: int, world: int, local: int, clock_sampler: Callable, timed: Callable,
               kernel_table: Callable | None = None) -> dict:
    from .. import components  # noqa: F401
    from ..algorithms.affinity_seg import AffinitySegmentation
    from ..engine.config import TrainerConfig
    from ..engine.graph_step import FlatParameters
    from ..engine.optimizer import build_optimizer
    from ..models.dinov3_vit3d import DinoVisionTransformer3D
    from ..ops import _native
    from ..ops.optim import clip_coefficient, grad_sumsq
    from ..ops.tp import TpComm
    from ..parallel.sequence_parallel import SequenceParallel, sync_partial_grads
    from ..parallel.tensor_parallel import apply_tensor_parallel, is_tensor_parallel
    from .windowed_tp import _groups

    _native.native()
    dev = torch.device("cuda", local)
    tp = min(2, world)
    tp_group, dp_group, dp_rank = _groups(world, tp) if world > 1 else (None, None, 0)
    torch.manual_seed(0)
    model = DinoVisionTransformer3D(**MODEL)
    alg = AffinitySegmentation(model, input_axes="lcxyz", offsets="nisb12", decoder="subpixel",
                               split_disconnected=False).to(dev)
    if world > 1:
        for p in alg.parameters():
            dist.broadcast(p.data, 0)
    comm = None
    if tp > 1:
        apply_tensor_parallel(model.tensor_parallel_plan(), tp_group)
        comm = TpComm(tp_group, args.tp_comm)
        model.enable_sequence_parallel(SequenceParallel(comm))
    flat = FlatParameters(alg)
    tcfg = TrainerConfig(max_steps=args.warmup + 2 * args.steps + 8, batch_size=BATCH, lr=1e-4, weight_decay=0.05,
                         warmup_steps=2, precision="bf16", grad_clip_norm=1.0, fused_optimizer="on")
    opt = build_optimizer(alg, tcfg)
    sharded = [p for m in alg.modules() if is_tensor_parallel(m) for name, p in m.named_parameters(recurse=False)
               if p.requires_grad and (name == "weight" or m._tp_mode != "row")]
    sharded_ids = {id(p) for p in sharded}
    replicated = [p for p in alg.parameters() if p.requires_grad and id(p) not in sharded_ids]

    imgs, labs = make_samples(2 * BATCH, seed=dp_rank + 1)
    imgs_dev, labs_dev = imgs.to(dev), labs.to(dev)
    imgs_pin, labs_pin = imgs.pin_memory(), labs.pin_memory()

    def step(img: torch.Tensor, lab: torch.Tensor) -> torch.Tensor:
        flat.grad.zero_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = alg({"img": img, "label": lab})
        out["loss"].backward()
        alg.zero_grad(set_to_none=True)
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

    def dev_batch(i: int):
        j = (i % 2) * BATCH
        return imgs_dev[j:j + BATCH], labs_dev[j:j + BATCH]

    for i in range(args.warmup):
        step(*dev_batch(i))
    torch.cuda.synchronize()
    if getattr(args, "profile_kernels", 0) and kernel_table is not None:
        table = kernel_table(lambda: step(*dev_batch(0)) and None, args.profile_kernels)
        if rank == 0:
            print(table, flush=True)
    ms, loss, clocks = timed(lambda i: step(*dev_batch(i)), args.steps, clock_sampler)
    e2e = None
    h2d = BATCH * SIDE**3 * (2 + 4)
    if not args.no_e2e:
        def e2e_step(i: int) -> torch.Tensor:
            j = (i % 2) * BATCH
            img = imgs_pin[j:j + BATCH].to(dev, non_blocking=True)
            lab = labs_pin[j:j + BATCH].to(dev, non_blocking=True)
            loss_i = step(img, lab)
            _ = loss_i.item()
            return loss_i

        e2e_ms, _, _ = timed(e2e_step, args.steps, None)
        e2e = {"ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "api": "mia_train_b200 affinity_seg + sequence-parallel dinov3_vit3d (eager step)"}
    errors = int(_native.native().check_errors(local))
    fwd = model.flops((1, SIDE, SIDE, SIDE)) * BATCH
    if comm is not None:
        comm.release()
    return {"ms": ms, "loss": float(loss), "clocks": clocks, "e2e": e2e, "errors": errors, "flops": 3.0 * fwd / tp,
            "global_batch": BATCH * (world // tp), "lib": _native.loaded_library_path(),
            "parallelism": f"tp{tp} x dp{world // tp} ({args.tp_comm if tp > 1 else 'no TP'})"}


def reference_arm(args: Any, rank: int, world: int, local: int, clock_sampler: Callable, timed: Callable,
                  repo: Path) -> dict:
    ref_root = repo / "baseline" / "_ref"
    if not (ref_root / "engine" / "trainer.py").is_file():
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    from algorithms.affinity_seg import AffinitySegmentation as RefAffinity  # type: ignore
    from data.base import BaseDataset as RefBase  # type: ignore
    from distributed.parallel_dims import ParallelDims  # type: ignore
    from engine.config import TrainerConfig as RefTrainerConfig  # type: ignore
    from engine.trainer import Trainer as RefTrainer  # type: ignore
    from models.dinov3_vit3d import DinoVisionTransformer3D as RefDino  # type: ignore

    dev = torch.device("cuda", local)
    imgs, labs = make_samples(2 * BATCH, seed=rank + 1)

    class SyntheticVoronoi(RefBase):
        def build_dataset(self):
            return torch.utils.data.TensorDataset(imgs.float(), labs)

        @property
        def sample_axes(self):
            return "lcxyz"

    torch.manual_seed(0)
    model = RefDino(**MODEL)
    ds = SyntheticVoronoi()
    alg = RefAffinity(model, ds, decoder="subpixel", split_disconnected=False)
    tcfg = RefTrainerConfig(max_steps=args.warmup + 2 * args.steps + 8, batch_size=BATCH, lr=1e-4, weight_decay=0.05,
                            warmup_steps=2, precision="bf16", grad_clip_norm=1.0, measure_mfu=False)
    dims = ParallelDims(dp_shard=world) if world > 1 else ParallelDims()
    mesh = dims.build_mesh("cuda") if world > 1 else None
    trainer = RefTrainer(alg, ds, tcfg, Path("/tmp") / f"ref_c5_{os.getpid()}", dims=dims, mesh=mesh, device=dev)

    def step(img: torch.Tensor, lab: torch.Tensor) -> torch.Tensor:
        with trainer._autocast():
            metrics = trainer.algorithm({"img": img.float(), "label": lab})
        metrics["loss"].backward()
        torch.nn.utils.clip_grad_norm_(trainer.algorithm.parameters(), tcfg.grad_clip_norm)
        trainer.optimizer.step()
        trainer.scheduler.step()
        trainer.optimizer.zero_grad(set_to_none=True)
        return metrics["loss"]

    imgs_dev, labs_dev = imgs.to(dev), labs.to(dev)
    imgs_pin, labs_pin = imgs.pin_memory(), labs.pin_memory()

    def dev_batch(i: int):
        j = (i % 2) * BATCH
        return imgs_dev[j:j + BATCH], labs_dev[j:j + BATCH]

    for i in range(args.warmup):
        step(*dev_batch(i))
    torch.cuda.synchronize()
    ms, loss, clocks = timed(lambda i: step(*dev_batch(i)), args.steps, clock_sampler)
    e2e = None
    if not args.no_e2e:
        def e2e_step(i: int) -> torch.Tensor:
            j = (i % 2) * BATCH
            loss_i = step(imgs_pin[j:j + BATCH].to(dev, non_blocking=True), labs_pin[j:j + BATCH].to(dev, non_blocking=True))
            _ = loss_i.item()
            return loss_i

        e2e_ms, _, _ = timed(e2e_step, args.steps, None)
        e2e = {"ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": BATCH * SIDE**3 * (2 + 4), "d2h_bytes_per_step": 4,
               "api": "reference Trainer objects, eager step"}
    from ..models.dinov3_vit3d import DinoVisionTransformer3D

    with torch.device("meta"):
        meta = DinoVisionTransformer3D(**MODEL)
    fwd = meta.flops((1, SIDE, SIDE, SIDE)) * BATCH
    return {"ms": ms, "loss": float(loss), "clocks": clocks, "e2e": e2e, "flops": 3.0 * fwd, "global_batch": BATCH * world,
            "parallelism": f"FSDP2 dp_shard={world}, 6 affinity channels (the reference's fixed layout)"}
