"""Worker for test_tp_multi.py (run under torch.distributed.run on 2 GPUs).

Builds the same windowed DINOv3 3-D backbone on every rank, keeps an unsharded copy as the oracle,
shards the other with the model's tensor-parallel plan (head-aligned qkv, column / row-parallel
MLP) and runs one bf16 forward + backward of both on the same input. The first argument picks the
TP communication: `allreduce` (replicated activations, NCCL all-reduces; SwiGLU MLP), `collective`
(sequence-parallel on NCCL collectives) or `fused` (sequence-parallel on the fused all-gather ->
GEMM and GEMM -> reduce-scatter kernels over NVLink peer memory); the sequence-parallel modes use
the GELU MLP and synchronise the per-shard norm / LayerScale gradients after backward. Rank 0 prints one JSON line:
the two losses, the largest relative gradient error of the replicated parameters (full gradient
on every rank in the Megatron form) and of the gathered sharded gradients, as ||g - g_ref|| / ||g_ref||,
the worst parameters by name, and whether the gathered state dict equals the oracle's exactly.
"""

from __future__ import annotations

import copy
import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D  # noqa: E402
from mia_train_b200.ops import _native  # noqa: E402
from mia_train_b200.ops.tp import TpComm  # noqa: E402
from mia_train_b200.parallel.sequence_parallel import SequenceParallel, sync_partial_grads  # noqa: E402
from mia_train_b200.parallel.tensor_parallel import apply_tensor_parallel, is_tensor_parallel  # noqa: E402


def _loss(model: torch.nn.Module, x: torch.Tensor, w: torch.Tensor, wc: torch.Tensor) -> torch.Tensor:
    # Linear in the normalised outputs: a squared norm of a LayerNorm output is nearly constant, so
    # its input gradient would be a cancellation that bf16 rounding dominates.
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model.forward_features(x)
    return (out["x_norm_patchtokens"].float() * w).sum() + (out["x_norm_clstoken"].float() * wc).sum()


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    _native.native()
    mode = sys.argv[1] if len(sys.argv) > 1 else "allreduce"
    torch.manual_seed(0)
    dense = DinoVisionTransformer3D(img_size=32, patch_size=4, embed_dim=256, depth=2, num_heads=8,
                                    n_storage_tokens=4, ffn_layer="swiglu" if mode == "allreduce" else "mlp",
                                    layerscale_init=0.1, window_size=4, global_every=2).to(dev)
    full_sd = {k: v.detach().clone() for k, v in dense.state_dict().items()}
    tp = copy.deepcopy(dense)
    n_sharded = apply_tensor_parallel(tp.tensor_parallel_plan(), dist.group.WORLD)
    comm = None
    if mode != "allreduce":
        comm = TpComm(dist.group.WORLD, mode)
        tp.enable_sequence_parallel(SequenceParallel(comm))
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(2, 1, 32, 32, 32, device=dev, generator=g)
    w = torch.randn(2, 512, 256, device=dev, generator=g)
    wc = torch.randn(2, 256, device=dev, generator=g)
    ref = _loss(dense, x, w, wc)
    ref.backward()
    for _ in range(2):  # the second pass re-runs every launch on the other workspace parity
        tp.zero_grad(set_to_none=True)
        loss = _loss(tp, x, w, wc)
        loss.backward()
    if comm is not None:
        sync_partial_grads(tp)

    dense_params = dict(dense.named_parameters())
    grad_rel = 0.0
    shard_rel = 0.0
    per_param: list[tuple[float, float, str, float]] = []  # (norm rel err, max rel err, name, ref norm)
    for name, p in tp.named_parameters():
        if p.grad is None:
            continue
        rg = dense_params[name].grad.float()
        mod = tp.get_submodule(name.rsplit(".", 1)[0]) if "." in name else tp
        if is_tensor_parallel(mod) and p.shape != dense_params[name].shape:
            # compare against the gathered full gradient
            parts = [torch.empty_like(p.grad) for _ in range(world)]
            dist.all_gather(parts, p.grad.contiguous())
            tp_mode = mod._tp_mode
            if tp_mode == "qkv":
                per = p.shape[0] // 3
                full = torch.cat([parts[r][q * per:(q + 1) * per] for q in range(3) for r in range(world)])
            elif tp_mode == "column" or p.dim() == 1:
                full = torch.cat(parts, dim=0)
            else:
                full = torch.cat(parts, dim=1)
            err = float((full.float() - rg).norm() / (rg.norm() + 1e-6))
            shard_rel = max(shard_rel, err)
            per_param.append((err, float((full.float() - rg).abs().max() / (rg.abs().max() + 1e-6)), name,
                              float(rg.norm())))
        else:
            err = float((p.grad.float() - rg).norm() / (rg.norm() + 1e-6))
            grad_rel = max(grad_rel, err)
            per_param.append((err, float((p.grad.float() - rg).abs().max() / (rg.abs().max() + 1e-6)), name,
                              float(rg.norm())))
    sd = tp.state_dict()
    sd_diff = max(float((sd[k].float() - v.float()).abs().max()) for k, v in full_sd.items())
    errors = int(_native.native().check_errors(local))
    if rank == 0:
        worst = sorted(per_param, reverse=True)[:6]
        print(json.dumps({"mode": mode, "loss": float(loss), "ref": float(ref), "grad_rel": grad_rel, "shard_rel": shard_rel,
                          "sd_diff": sd_diff, "sharded_layers": n_sharded, "errors": errors,
                          "worst": [[round(a, 4), round(m, 4), n, round(r, 6)] for a, m, n, r in worst]}),
              flush=True)
    dist.barrier()
    if comm is not None:
        comm.release()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
