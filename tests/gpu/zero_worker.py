"""Worker for test_zero_multi.py (run under torch.distributed.run on 2+ GPUs).

Trains a small bf16 MAE for a few captured steps with each data-parallel gradient path and prints
one JSON line (rank 0) with the largest parameter difference between paths and the losses.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

from mia_train_b200.algorithms.mae import MAE  # noqa: E402
from mia_train_b200.engine.config import TrainerConfig  # noqa: E402
from mia_train_b200.engine.graph_step import CapturedStep  # noqa: E402
from mia_train_b200.engine.optimizer import build_lr_scheduler, build_optimizer  # noqa: E402
from mia_train_b200.models.vit import ViT3D  # noqa: E402
from mia_train_b200.ops import _native  # noqa: E402


def train(impl: str, rank: int, dev: torch.device, steps: int) -> tuple[list[torch.Tensor], list[float]]:
    overlap = not impl.endswith("_serial")
    impl = impl.removesuffix("_serial")
    wire = "fp32" if impl.endswith("_fp32") else "bf16"
    impl = impl.removesuffix("_fp32")
    torch.manual_seed(0)
    model = ViT3D(img_size=(32, 32, 32), patch_size=(8, 8, 8), embed_dim=128, depth=2, num_heads=4)
    alg = MAE(model, input_axes="lcxyz", decoder_embed_dim=64, decoder_depth=1, decoder_num_heads=4).to(dev)
    cfg = TrainerConfig(max_steps=steps + 4, batch_size=2, lr=1e-3, warmup_steps=1, precision="bf16",
                        grad_clip_norm=1.0, fused_optimizer="on")
    opt = build_optimizer(alg, cfg)
    build_lr_scheduler(opt, cfg)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    batches = [torch.randn(2, 1, 1, 32, 32, 32, device=dev, generator=g) for _ in range(steps)]
    step = CapturedStep(alg, opt, cfg, {"img": batches[0]}, eager_steps=2, process_group=dist.group.WORLD,
                        dp_impl=impl, overlap=overlap, dp_wire=wire)
    losses = []
    for b in batches:
        m = step({"img": b})
        losses.append(float(m["loss"]))
    torch.cuda.synchronize()
    step.release()
    return [p.detach().float().clone() for p in alg.parameters()], losses


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank = dist.get_rank()
    _native.native()
    steps = 5
    impls = ("allreduce", "nccl", "p2p", "p2p_serial", "p2p_fp32")
    results = {impl: train(impl, rank, dev, steps) for impl in impls}
    ref, _ = results["allreduce"]
    diffs = {}
    for impl in impls[1:]:
        params, _ = results[impl]
        diffs[impl] = max(float((a - b).abs().max() / (b.abs().max() + 1e-12)) for a, b in zip(params, ref, strict=True))
    # replicas must agree exactly with each other after the final gather
    p2p_params, _ = results["p2p"]
    flat = torch.cat([p.flatten() for p in p2p_params])
    gathered = [torch.empty_like(flat) for _ in range(dist.get_world_size())]
    dist.all_gather(gathered, flat)
    replica_diff = max(float((x - gathered[0]).abs().max()) for x in gathered)
    errors = int(_native.native().check_errors(local))
    if rank == 0:
        print(json.dumps({"rel_diff": diffs, "replica_diff": replica_diff, "errors": errors,
                          "losses": {k: v[1] for k, v in results.items()}}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
