"""DINOv3 self-distillation of a ViT-H-class 3D encoder under data parallelism (the `bench.py
--config dinov3_dp` workload).

Workload: `dinov3_vit3d` dim 1280 / depth 32 / 20 heads / GELU MLP 5120, patch 16^3, 3D RoPE, 4
register tokens; the `dinov3` objective with DINO and iBOT heads of 65536 prototypes (bottleneck
256, hidden 2048, 3 layers), Sinkhorn-Knopp centring (3 iterations), KoLeo weight 0.1, iBOT mask
ratio U[0.1, 0.5] on half of the global views, teacher EMA momentum 0.994 -> 1.0; per GPU 8
samples, each giving 2 global crops of 128^3 (512 patch tokens) and 8 local crops of 64^3 (64 patch
tokens), cut from 192^3 volumes with random flips and an intensity jitter (contrast scale
U[0.8, 1.2], brightness shift of at most 0.1; no blur, noise or rotation); bf16 autocast; AdamW
(lr 5e-4, wd 0.04), grad clip 3.0.

Data: the same uint8 generator as the MAE benchmark (blurred Gaussian noise plus bright ellipsoid
blobs) at 192^3, z-scored on the device inside the step.

* native arm: this framework's `DINOv3` (native soft-target cross-entropy, KoLeo, Sinkhorn with the
  teacher heads' column sums from the prototype GEMM epilogue, native EMA of the teacher after every
  optimizer step), data parallel over N GPUs: flat fp32 gradient buffer all-reduced, clip, fused
  AdamW.
* reference arm: the unmodified reference (baseline/_ref) through its own Trainer, model and
  algorithm objects on FSDP2 dp_shard = N with the same per-GPU batch and crop settings. The
  reference's engine never calls `update_teacher`, so its step has no EMA cost; its teacher stays
  the initial student.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path
from typing import Any, Callable

import torch
import torch.distributed as dist

MODEL = dict(img_size=128, patch_size=16, embed_dim=1280, depth=32, num_heads=20, ffn_ratio=4.0,
             n_storage_tokens=4)
SIDE = 192
BATCH = 8
ALG = dict(global_crop_size=128, local_crop_size=64, n_local_crops=8, head_n_prototypes=65536,
           head_bottleneck_dim=256, head_hidden_dim=2048, head_nlayers=3, momentum_teacher=0.994,
           final_momentum_teacher=1.0, koleo_loss_weight=0.1, mask_ratio_min_max=(0.1, 0.5),
           augmentation=dict(brightness=0.1, contrast=0.2, intensity_prob=1.0, blur_prob=0.0, noise_prob=0.0,
                             flip_prob=0.5, rotate_prob=0.0))
METRIC = ("samples/sec (dinov3 ViT-H-class 3D, 2x128^3 + 8x64^3 crops, 65536 prototypes, bf16), whole box, "
          "device-timed max over ranks")
DATA = "synthetic (uint8 blurred-noise + ellipsoid 192^3 volumes, z-scored on device; random-init weights)"
SEQ_LEN = 517  # a global crop: 512 patch tokens + class token + 4 registers


def describe(n_gpus: int) -> dict:
    return {
        "model": "dinov3_vit3d ViT-H-class (1280/32/20, MLP 5120, 4 registers) + dinov3 (DINO + iBOT heads of "
                 "65536 prototypes, Sinkhorn 3 iterations, KoLeo 0.1, EMA teacher)",
        "img": "192^3 volumes -> 2 global crops 128^3 + 8 local crops 64^3 per sample, patch 16",
        "per_gpu_batch": BATCH,
    }


def make_volumes(n: int, seed: int) -> torch.Tensor:
    from .windowed_tp import make_volumes as mk

    return mk(n, seed, side=SIDE)


def _step_flops(model: Any) -> float:
    """Per-GPU FLOPs of one step: teacher forward on the global crops, student forward and backward
    (2x) on global and local crops, and the heads' matmuls (prototype layer included) on the class
    tokens and the expected number of masked patch tokens."""
    g, l = ALG["global_crop_size"], ALG["local_crop_size"]
    fg = model.flops((1, g, g, g))
    fl = model.flops((1, l, l, l))
    d, h, bn = model.embed_dim, ALG["head_hidden_dim"], ALG["head_bottleneck_dim"]
    head_macs = d * h + h * h + h * bn + bn * ALG["head_n_prototypes"]
    n_masked = 0.5 * 0.3 * (g // model.patch_size) ** 3  # expected masked patches per global view
    n_loc = ALG["n_local_crops"]
    teacher = BATCH * (2 * fg + 2 * head_macs * 2 * (1 + n_masked))
    student = BATCH * (2 * fg + n_loc * fl + 2 * head_macs * (2 + n_loc + 2 * n_masked))
    return teacher + 3.0 * student


def native_arm(args: Any, rank: int, world: int, local: int, clock_sampler: Callable, timed: Callable,
               kernel_table: Callable | None = None) -> dict:
    from .. import components  # noqa: F401
    from ..algorithms.dinov3_ssl import DINOv3
    from ..engine.config import TrainerConfig
    from ..engine.graph_step import FlatParameters
    from ..engine.optimizer import build_optimizer
    from ..models.dinov3_vit3d import DinoVisionTransformer3D
    from ..ops import _native
    from ..ops.data import zscore_u8
    from ..ops.optim import clip_coefficient, grad_sumsq

    _native.native()
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    model = DinoVisionTransformer3D(**MODEL)
    alg = DINOv3(model, input_axes="lcxyz", total_steps=10_000, **ALG).to(dev)
    if world > 1:
        for p in alg.parameters():
            dist.broadcast(p.data, 0)
    flat = FlatParameters(alg)
    tcfg = TrainerConfig(max_steps=args.warmup + 2 * args.steps + 8, batch_size=BATCH, lr=5e-4, weight_decay=0.04,
                         beta1=0.9, beta2=0.999, warmup_steps=2, precision="bf16", grad_clip_norm=3.0,
                         fused_optimizer="on")
    opt = build_optimizer(alg, tcfg)
    params = [p for p in alg.parameters() if p.requires_grad]
    torch.cuda.manual_seed(1234 + rank)

    pool_cpu = make_volumes(2 * BATCH, seed=rank + 1)
    pool_dev = pool_cpu.to(dev)
    pool_pinned = pool_cpu.pin_memory()
    step_no = [0]

    def step(u8: torch.Tensor) -> torch.Tensor:
        flat.grad.zero_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = alg({"img": zscore_u8(u8, torch.bfloat16)})
        out["loss"].backward()
        alg.zero_grad(set_to_none=True)  # every gradient is in the flat buffer (main_grad) now
        if world > 1:
            dist.all_reduce(flat.grad)
        sq = grad_sumsq([p.main_grad for p in params])
        opt.grad_scale = clip_coefficient(sq.sqrt() / world, 3.0) / world
        opt.step()
        step_no[0] += 1
        alg.after_optimizer_step(step_no[0])
        return out["loss"]

    def batch(i: int) -> torch.Tensor:
        j = (i % 2) * BATCH
        return pool_dev[j:j + BATCH]

    for i in range(args.warmup):
        step(batch(i))
    torch.cuda.synchronize()
    if getattr(args, "profile_kernels", 0) and kernel_table is not None:
        table = kernel_table(lambda: step(batch(0)) and None, args.profile_kernels)
        if rank == 0:
            print(table, flush=True)
    ms, loss, clocks = timed(lambda i: step(batch(i)), args.steps, clock_sampler)
    e2e = None
    if not args.no_e2e:
        def e2e_step(i: int) -> torch.Tensor:
            j = (i % 2) * BATCH
            loss_i = step(pool_pinned[j:j + BATCH].to(dev, non_blocking=True))
            _ = loss_i.item()
            return loss_i

        e2e_ms, _, _ = timed(e2e_step, args.steps, None)
        e2e = {"ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": BATCH * SIDE**3, "d2h_bytes_per_step": 4,
               "api": "mia_train_b200 DINOv3 + dinov3_vit3d (eager step)"}
    errors = int(_native.native().check_errors(local))
    return {"ms": ms, "loss": float(loss), "clocks": clocks, "e2e": e2e, "errors": errors,
            "flops": _step_flops(model), "global_batch": BATCH * world, "lib": _native.loaded_library_path(),
            "parallelism": f"dp{world} (flat gradient all-reduce, fused AdamW, native EMA teacher)",
            "memory_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1)}


def reference_arm(args: Any, rank: int, world: int, local: int, clock_sampler: Callable, timed: Callable,
                  repo: Path) -> dict:
    ref_root = repo / "baseline" / "_ref"
    if not (ref_root / "engine" / "trainer.py").is_file():
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    from algorithms.dinov3_ssl import DINOv3 as RefDINOv3  # type: ignore
    from data.base import BaseDataset as RefBase  # type: ignore
    from distributed.parallel_dims import ParallelDims  # type: ignore
    from engine.config import TrainerConfig as RefTrainerConfig  # type: ignore
    from engine.trainer import Trainer as RefTrainer  # type: ignore
    from models.dinov3_vit3d import DinoVisionTransformer3D as RefDino  # type: ignore

    dev = torch.device("cuda", local)
    pool = make_volumes(2 * BATCH, seed=rank + 1)

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
    alg = RefDINOv3(model, ds, total_steps=10_000, **ALG)
    tcfg = RefTrainerConfig(max_steps=args.warmup + 2 * args.steps + 8, batch_size=BATCH, lr=5e-4, weight_decay=0.04,
                            beta1=0.9, beta2=0.999, warmup_steps=2, precision="bf16", grad_clip_norm=3.0,
                            measure_mfu=False)
    dims = ParallelDims(dp_shard=world) if world > 1 else ParallelDims()
    mesh = dims.build_mesh("cuda") if world > 1 else None
    trainer = RefTrainer(alg, ds, tcfg, Path("/tmp") / f"ref_c3_{os.getpid()}", dims=dims, mesh=mesh, device=dev)

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

    def batch(i: int) -> torch.Tensor:
        j = (i % 2) * BATCH
        return pool_dev[j:j + BATCH]

    for i in range(args.warmup):
        step(batch(i))
    torch.cuda.synchronize()
    ms, loss, clocks = timed(lambda i: step(batch(i)), args.steps, clock_sampler)
    e2e = None
    if not args.no_e2e:
        def e2e_step(i: int) -> torch.Tensor:
            j = (i % 2) * BATCH
            loss_i = step(pool_pinned[j:j + BATCH].to(dev, non_blocking=True))
            _ = loss_i.item()
            return loss_i

        e2e_ms, _, _ = timed(e2e_step, args.steps, None)
        e2e = {"ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": BATCH * SIDE**3, "d2h_bytes_per_step": 4,
               "api": "reference Trainer objects, eager step"}
    from ..models.dinov3_vit3d import DinoVisionTransformer3D

    with torch.device("meta"):
        meta = DinoVisionTransformer3D(**MODEL)
    return {"ms": ms, "loss": float(loss), "clocks": clocks, "e2e": e2e, "flops": _step_flops(meta),
            "global_batch": BATCH * world, "parallelism": f"FSDP2 dp_shard={world} (no teacher EMA in its engine)"}
