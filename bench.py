"""Throughput benchmark: ViT-L 3D MAE (128^3 volumes, patch 16^3, 512 tokens), bf16, per-rank batch 16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload (the same for both arms): `vit3d` encoder dim 1024 / depth 24 / 16 heads / MLP 4096 on
single-channel 128^3 volumes with patch 16^3; `mae` with mask ratio 0.75, decoder dim 512 /
depth 8 / 16 heads, norm-pix MSE; AdamW (lr 1.5e-4, betas 0.9/0.95, wd 0.05) with a cosine
schedule, grad clip 1.0, bf16 autocast, no activation checkpointing. Data are synthetic: uint8
volumes of blurred Gaussian noise (sigma 3 voxels) plus Poisson(50) bright ellipsoids (radii 2-8),
z-scored per volume, random-init weights.

`value` is whole-job samples/s from CUDA-event timing of exactly K steps (max over ranks), bracketed
by a barrier and a synchronize; the batch, weights and activations are far larger than the 126 MB
L2, so no flush is needed. `e2e` is the same metric through the framework's public step API with a
pinned host->device copy of each step's batch and a device->host read of each step's loss.

Both arms receive the same uint8 volumes (16 MiB per step per rank over PCIe) and z-score them on
the device inside the timed step. Native arm: this framework (native sm_100a kernels, one CUDA
graph per step, fused AdamW; with N > 1 a sharded optimizer over peer memory). Reference arm: the
unmodified reference package installed in baseline/_ref, driven through its own
Trainer/algorithm/optimizer objects and its stock eager step (FSDP2 dp_shard = N when N > 1).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

CONFIG = {
    "model": "vit3d ViT-L (1024/24/16, MLP 4096) + mae (mask 0.75, decoder 512/8/16)",
    "img_size": 128,
    "patch": 16,
    "seq_len": 512,
    "per_rank_batch": 16,
}
METRIC = "samples/sec (MAE ViT-L 3D, 128^3, patch 16, bf16), whole box, device-timed max over ranks"
PEAK_BF16 = 2250e12  # dense bf16 per GPU, the MFU denominator used by the reference's table


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--batch", type=int, default=CONFIG["per_rank_batch"])
    ap.add_argument("--depth", type=int, default=24, help="encoder depth (24 = the named config)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--overlap-dp", action="store_true",
                    help="reduce-scatter each block's gradients during backward (side stream) instead of after it")
    ap.add_argument("--dp-impl", choices=("p2p", "nccl", "allreduce"), default="p2p",
                    help="data-parallel gradient path for N > 1 (sharded optimizer over peer memory by default)")
    ap.add_argument("--profile-kernels", type=int, default=0, metavar="STEPS",
                    help="also profile STEPS eager steps and print the per-kernel device-time table")
    ap.add_argument("--config", choices=("vit_l_mae", "windowed_tp", "affinity_tp", "dinov3_dp"), default="vit_l_mae",
                    help="vit_l_mae: ViT-L 3D MAE at 128^3 (the default headline workload); windowed_tp: windowed "
                         "dinov3_vit3d ViT-L SimMIM at 256^3 / patch 8 under sequence-parallel TP (TP = min(4, N)); "
                         "affinity_tp: ViT-L affinity segmentation, 128^3 / patch 8, 12 offsets (TP = min(2, N)); "
                         "dinov3_dp: DINOv3 on a ViT-H-class 3D encoder, 8 samples of 2 + 8 crops per GPU")
    ap.add_argument("--tp-comm", choices=("fused", "collective"), default="fused",
                    help="windowed_tp: fused collective-GEMM kernels over NVLink, or NCCL collectives")
    return ap.parse_args()


def dist_setup() -> tuple[int, int, int]:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        return dist.get_rank(), world, local
    return 0, 1, local


def make_pool(n: int, seed: int) -> torch.Tensor:
    """n uint8 volumes (n, 1, 1, 128, 128, 128): blurred noise + ellipsoid blobs (before z-scoring)."""
    from mia_train_b200.data.synthetic import blobs_volume

    vols = []
    for i in range(n):
        g = torch.Generator().manual_seed(seed * 1000 + i)
        v = blobs_volume((128, 128, 128), 3.0, 50.0, (2.0, 8.0), g)
        # blobs_volume z-scores; store the uint8 form the config specifies and z-score on device
        u8 = ((v - v.min()) / (v.max() - v.min()).clamp_min(1e-6) * 255).round().to(torch.uint8)
        vols.append(u8)
    return torch.stack(vols)[:, None, None].contiguous()


def zscore_u8_torch(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Per-volume z-score of a uint8 batch (B, L, C, X, Y, Z) in torch ops (the reference arm)."""
    v = x.float()
    dims = tuple(range(1, v.dim()))
    mean = v.mean(dim=dims, keepdim=True)
    std = v.std(dim=dims, keepdim=True).clamp_min(1e-6)
    return ((v - mean) / std).to(dtype)


class ClockSampler:
    """Samples SM clocks and throttle reasons while the timed region runs (read-only queries).

    NVML is polled every 10 ms from a thread (the timed region of a default run is a few tenths of
    a second, too short for `nvidia-smi`'s ~200 ms cadence); the device is matched to the CUDA
    device by PCI bus id. Falls back to `nvidia-smi` polling when NVML is unavailable.
    """

    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, cuda_index: int, period_s: float = 0.01) -> None:
        self.cuda_index = cuda_index
        self.period_s = period_s
        self.samples: list[tuple[float, float | None, tuple[str, ...]]] = []  # (sm MHz, max MHz, reasons)
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self.source = "nvml"

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001 - domain formatting differs between drivers
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus[4:])

    def _run(self) -> None:
        try:
            nv, handle = self._nvml_handle()
            bits = {
                "hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
            }
            max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM))
            while not self._stop.is_set():
                sm = float(nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(handle)
                self.samples.append((sm, max_mhz, tuple(k for k, b in bits.items() if mask & b)))
                self._stop.wait(self.period_s)
        except Exception:  # noqa: BLE001
            self.source = "nvidia-smi"
            self._run_smi()

    def _run_smi(self) -> None:
        fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--id={self.cuda_index}", f"--query-gpu={fields}", "--format=csv,noheader,nounits"],
                    capture_output=True, text=True, timeout=5,
                ).stdout.strip()
                v = [x.strip() for x in out.split(",")]
                if len(v) >= 6 and v[0].replace(".", "").isdigit():
                    reasons = tuple(n for n, x in zip(self.REASONS, v[2:6], strict=True) if x == "Active")
                    self.samples.append((float(v[0]), float(v[1]) if v[1].replace(".", "").isdigit() else None, reasons))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.2)

    def __enter__(self) -> ClockSampler:
        self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        self._thread.join(timeout=6)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = sorted(s[0] for s in self.samples)
        mx = max((s[1] for s in self.samples if s[1] is not None), default=None)
        reasons = sorted({r for s in self.samples for r in s[2]})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": reasons, "samples": len(self.samples),
                "source": self.source}


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()


# ------------------------------------------------------------------------------------------ native
def native_arm(args: argparse.Namespace, rank: int, world: int, local: int) -> dict:
    from mia_train_b200 import components  # noqa: F401
    from mia_train_b200.algorithms.mae import MAE
    from mia_train_b200.engine.config import TrainerConfig
    from mia_train_b200.engine.graph_step import CapturedStep
    from mia_train_b200.engine.mfu import measure_step_flops
    from mia_train_b200.engine.optimizer import build_lr_scheduler, build_optimizer
    from mia_train_b200.models.vit import ViT3D
    from mia_train_b200.ops import _native

    _native.native()  # fail loudly if the extension is missing
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    model = ViT3D(img_size=(128,) * 3, patch_size=(16,) * 3, embed_dim=1024, depth=args.depth, num_heads=16, mlp_ratio=4.0)
    alg = MAE(model, input_axes="lcxyz", mask_ratio=0.75, decoder_embed_dim=512, decoder_depth=8, decoder_num_heads=16)
    alg = alg.to(dev)
    if world > 1:  # identical initial weights on every rank
        for p in alg.parameters():
            dist.broadcast(p.data, 0)
    total_steps = args.warmup + 2 * args.steps + 8
    tcfg = TrainerConfig(
        max_steps=total_steps, batch_size=args.batch, lr=1.5e-4, weight_decay=0.05, beta1=0.9, beta2=0.95,
        warmup_steps=2, lr_schedule="cosine", precision="bf16", grad_clip_norm=1.0, fused_optimizer="on",
    )
    opt = build_optimizer(alg, tcfg)
    build_lr_scheduler(opt, tcfg)  # records initial_lr per group, as the Trainer does

    pool_cpu = make_pool(2 * args.batch, seed=rank + 1)
    pool_pinned = pool_cpu.pin_memory()
    pool_dev = pool_cpu.to(dev)

    from mia_train_b200.ops.data import zscore_u8  # native per-volume z-score (uint8 -> bf16)

    def forward(batch):
        return alg({"img": zscore_u8(batch["img"], torch.bfloat16)})

    # FLOPs of one step on this rank, counted in PyTorch math (the counter cannot see custom kernels)
    probe = {"img": pool_dev[: args.batch]}
    step_flops = measure_step_flops(alg, {"img": zscore_u8(probe["img"], torch.float32)},
                                    lambda: torch.autocast("cuda", dtype=torch.bfloat16))

    step = CapturedStep(alg, opt, tcfg, {"img": pool_dev[: args.batch]}, eager_steps=2, forward=forward,
                        process_group=dist.group.WORLD if world > 1 else None, dp_impl=args.dp_impl,
                        overlap=args.overlap_dp)

    def device_batch(i: int) -> dict:
        j = (i * args.batch) % pool_dev.shape[0]
        return {"img": pool_dev[j:j + args.batch]}

    def host_batch(i: int) -> dict:
        j = (i * args.batch) % pool_pinned.shape[0]
        return {"img": pool_pinned[j:j + args.batch]}

    # count this framework's kernel launches in one eager step (the replayed graph holds the same)
    launches = count_native_launches(lambda: step._body() and None, alg)
    if args.profile_kernels:  # every rank runs the profiled steps (they hold collectives)
        table = kernel_table(lambda: step._body() and None, args.profile_kernels)
        if rank == 0:
            print(table, flush=True)

    for i in range(args.warmup):
        step(device_batch(i))
    torch.cuda.synchronize()

    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(device_batch(i))
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    loss = float(step.static_metrics["loss"].item())
    errors = int(_native.native().check_errors(local))

    e2e = None
    if not args.no_e2e:
        barrier(world)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        step.prefetch(host_batch(0))
        s2.record()
        for i in range(args.steps):
            m = step()  # consumes the batch prefetched during the previous step
            step.prefetch(host_batch(i + 1))  # next batch: pinned host -> device, overlapping this step
            _ = m["loss"].item()  # device -> host read of the step's result
        step.wait_prefetch()  # the copy issued during the last step is part of the timed work
        e2.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(s2.elapsed_time(e2) / args.steps, world)
        h2d = args.batch * 128**3  # uint8 bytes per step per rank
        e2e = {"value": round(args.batch * world * 1000.0 / e2e_ms, 3), "unit": "samples/s",
               "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "api": "mia_train_b200.engine.graph_step.CapturedStep"}
    step.release()
    return {
        "ms": ms, "flops": step_flops, "loss": loss, "clocks": clocks.summary(), "e2e": e2e,
        "launches_per_step": launches, "errors": errors,
        "lib": _native.loaded_library_path(),
    }


def count_native_launches(fn, module) -> int | None:
    """Kernels of this framework's extension launched by `fn` (profiled once, eagerly)."""
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        mine = [n for n in names if "mia::" in n]
        module.zero_grad(set_to_none=True)
        return len(mine)
    except Exception:  # noqa: BLE001
        return None


def kernel_table(fn, steps: int) -> str:
    """Per-kernel device time of `steps` eager calls of `fn`, sorted by total time, with the share of
    device time spent in this framework's own kernels (`mia::`) against PyTorch / library kernels."""
    from collections import defaultdict

    from torch.profiler import ProfilerActivity, profile

    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            fn()
        torch.cuda.synchronize()
    agg: dict[str, list[float]] = defaultdict(lambda: [0.0, 0])
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            agg[e.name][0] += e.device_time_total / 1000.0
            agg[e.name][1] += 1
    total = sum(v[0] for v in agg.values()) / steps
    mine = sum(v[0] for k, v in agg.items() if "mia::" in k) / steps
    n_mine = sum(v[1] for k, v in agg.items() if "mia::" in k) // steps
    n_all = sum(v[1] for v in agg.values()) // steps
    rows = sorted(agg.items(), key=lambda kv: -kv[1][0])
    lines = [f"kernel table: {total:.3f} ms device time per step, {n_all} launches per step",
             f"  native (mia::) kernels: {mine:.3f} ms ({100 * mine / max(total, 1e-9):.1f}%), {n_mine} launches; "
             f"other (PyTorch / library): {total - mine:.3f} ms, {n_all - n_mine} launches"]
    for name, (ms, n) in rows[:40]:
        tag = "native" if "mia::" in name else "other "
        lines.append(f"  {ms / steps:8.3f} ms {100 * ms / steps / total:5.1f}%  x{n // steps:<4d} {tag} {name[:100]}")
    return "\n".join(lines)


# --------------------------------------------------------------------------------------- reference
def reference_arm(args: argparse.Namespace, rank: int, world: int, local: int) -> dict:
    ref_root = REPO / "baseline" / "_ref"
    if not (ref_root / "engine" / "trainer.py").is_file():
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    from algorithms.mae import MAE as RefMAE  # type: ignore
    from data.base import BaseDataset as RefBase  # type: ignore
    from distributed.parallel_dims import ParallelDims  # type: ignore
    from engine.config import TrainerConfig as RefTrainerConfig  # type: ignore
    from engine.trainer import Trainer as RefTrainer  # type: ignore
    from models.vit import ViT3D as RefViT3D  # type: ignore

    dev = torch.device("cuda", local)
    pool = make_pool(2 * args.batch, seed=rank + 1)  # uint8, as the native arm receives them
    vols = zscore_u8_torch(pool, torch.float32)  # the dataset object's float contract (not timed)

    class SyntheticVolumes(RefBase):
        """A synthetic dataset registered the way the reference's own tests do."""

        def build_dataset(self):
            return torch.utils.data.TensorDataset(vols)

        @property
        def sample_axes(self):
            return "lcxyz"

    torch.manual_seed(0)
    model = RefViT3D(img_size=(128,) * 3, patch_size=(16,) * 3, embed_dim=1024, depth=args.depth, num_heads=16, mlp_ratio=4.0)
    ds = SyntheticVolumes()
    alg = RefMAE(model, ds, mask_ratio=0.75, decoder_embed_dim=512, decoder_depth=8, decoder_num_heads=16)
    total_steps = args.warmup + 2 * args.steps + 8
    tcfg = RefTrainerConfig(
        max_steps=total_steps, batch_size=args.batch, lr=1.5e-4, weight_decay=0.05, beta1=0.9, beta2=0.95,
        warmup_steps=2, lr_schedule="cosine", precision="bf16", grad_clip_norm=1.0, measure_mfu=False,
    )
    dims = ParallelDims(dp_shard=world) if world > 1 else ParallelDims()
    mesh = dims.build_mesh("cuda") if world > 1 else None
    out_dir = Path("/tmp") / f"ref_bench_{os.getpid()}"
    trainer = RefTrainer(alg, ds, tcfg, out_dir, dims=dims, mesh=mesh, device=dev)

    def one_step(batch: dict) -> torch.Tensor:
        # the per-volume z-score of the uint8 batch (the same input work the native arm does on the
        # device), then the body of the reference's Trainer.train loop (src/engine/trainer.py:249-280)
        batch = {"img": zscore_u8_torch(batch["img"], torch.float32)}
        with trainer._autocast():
            metrics = trainer.algorithm(batch)
        metrics["loss"].backward()
        torch.nn.utils.clip_grad_norm_(trainer.algorithm.parameters(), tcfg.grad_clip_norm)
        trainer.optimizer.step()
        trainer.scheduler.step()
        trainer.optimizer.zero_grad(set_to_none=True)
        return metrics["loss"]

    vols_dev = pool.to(dev)
    vols_pinned = pool.pin_memory()

    def device_batch(i: int) -> dict:
        j = (i * args.batch) % vols_dev.shape[0]
        return {"img": vols_dev[j:j + args.batch]}

    for i in range(args.warmup):
        one_step(device_batch(i))
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            loss = one_step(device_batch(i))
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    e2e = None
    if not args.no_e2e:
        barrier(world)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            j = (i * args.batch) % vols_pinned.shape[0]
            batch = {"img": vols_pinned[j:j + args.batch].to(dev, non_blocking=True)}
            loss = one_step(batch)
            _ = loss.item()
        e2.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(s2.elapsed_time(e2) / args.steps, world)
        e2e = {"value": round(args.batch * world * 1000.0 / e2e_ms, 3), "unit": "samples/s",
               "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": args.batch * 128**3, "d2h_bytes_per_step": 4,
               "api": "reference Trainer objects, eager step"}
    # FLOPs with the reference's own counter (SDPA is visible to it)
    from engine.mfu import measure_step_flops as ref_flops  # type: ignore

    step_flops = ref_flops(trainer.algorithm, {"img": zscore_u8_torch(device_batch(0)["img"], torch.float32)},
                           trainer._autocast)
    return {"ms": ms, "flops": step_flops, "loss": float(loss.item()), "clocks": clocks.summary(), "e2e": e2e}


def timed_loop(fn, steps: int, sampler_index: int | None, world: int) -> tuple[float, float, dict | None]:
    """(ms per step, max over ranks; last loss; clock summary): CUDA events around exactly `steps`
    calls of fn(i), bracketed by a barrier and a synchronize on both sides."""
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(sampler_index) if sampler_index is not None else None
    if sampler is not None:
        sampler.__enter__()
    start.record()
    loss = None
    for i in range(steps):
        loss = fn(i)
    end.record()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.__exit__(None, None, None)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / steps, world)
    return ms, float(loss.item()) if loss is not None else float("nan"), sampler.summary() if sampler else None


EXTRA_CONFIGS = ("windowed_tp", "affinity_tp", "dinov3_dp")


def extra_config_main(args: argparse.Namespace, rank: int, world: int, local: int) -> None:
    """The benchmark workloads that live in `mia_train_b200.benchmarks` (one module per workload,
    each with `native_arm`, `reference_arm`, `describe` and its METRIC / DATA / SEQ_LEN)."""
    import importlib

    wtp = importlib.import_module(f"mia_train_b200.benchmarks.{args.config}")

    def timed(fn, steps, sampler):
        return timed_loop(fn, steps, local if sampler is not None else None, world)

    if args.impl == "reference":
        res = wtp.reference_arm(args, rank, world, local, ClockSampler, timed, REPO)
    else:
        res = wtp.native_arm(args, rank, world, local, ClockSampler, timed, kernel_table)
    if rank == 0:
        if "unavailable" in res:
            print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}), flush=True)
            return
        gb = res["global_batch"]
        value = gb * 1000.0 / res["ms"]
        line = {
            "metric": wtp.METRIC,
            "value": round(value, 3), "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(res["ms"], 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": wtp.DATA,
            "config": {**wtp.describe(world), "global_batch": gb,
                       "seq_len": wtp.SEQ_LEN,
                       "parallelism": res["parallelism"], "l2": "activations far larger than L2 (no flush)"},
            "mfu": round(res["flops"] / (res["ms"] / 1000.0) / PEAK_BF16, 4),
            "tflops_per_gpu": round(res["flops"] / (res["ms"] / 1000.0) / 1e12, 1),
            "loss": round(res["loss"], 5), "clocks": res["clocks"],
        }
        if res.get("e2e"):
            e = res["e2e"]
            line["e2e"] = {"value": round(gb * 1000.0 / e["ms_per_step"], 3), "unit": "samples/s", **e}
        if args.impl == "reference":
            line["impl"] = "reference"
        else:
            line["kernel_errors"] = res["errors"]
            line["native_library"] = res["lib"]
        if "memory_gb" in res:
            line["max_memory_allocated_gb"] = res["memory_gb"]
        print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    rank, world, local = dist_setup()
    if args.config in EXTRA_CONFIGS:
        extra_config_main(args, rank, world, local)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.impl == "reference":
        res = reference_arm(args, rank, world, local)
    else:
        res = native_arm(args, rank, world, local)
    if rank == 0:
        if "unavailable" in res:
            print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}), flush=True)
        else:
            value = args.batch * world * 1000.0 / res["ms"]
            mfu = res["flops"] / (res["ms"] / 1000.0) / PEAK_BF16
            line = {
                "metric": METRIC,
                "value": round(value, 3),
                "unit": "samples/s",
                "n_gpus": world,
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": round(res["ms"], 3),
                "higher_is_better": True,
                "scaling": "weak",
                "vs_baseline": None,
                "dtype": "bf16",
                "data": "synthetic (uint8 blurred-noise + ellipsoid volumes, z-scored on device; random-init weights)",
                "config": {
                    "model": CONFIG["model"] if args.depth == 24 else CONFIG["model"] + f" (depth {args.depth})",
                    "global_batch": args.batch * world,
                    "seq_len": CONFIG["seq_len"],
                    "parallelism": f"dp{world}" + (
                        f" (sharded optimizer, {args.dp_impl}{', overlapped' if args.overlap_dp else ''})"
                        if world > 1 and args.impl == "native" else ""),
                    "l2": "inputs and weights larger than L2 (no flush)",
                },
                "mfu": round(mfu, 4),
                "tflops_per_gpu": round(res["flops"] / (res["ms"] / 1000.0) / 1e12, 1),
                "step_tflop_per_rank": round(res["flops"] / 1e12, 4),
                "loss": round(res["loss"], 5),
                "clocks": res["clocks"],
                "e2e": res["e2e"],
            }
            if args.impl == "reference":
                line["impl"] = "reference"
            else:
                line["gpu_launches"] = (res["launches_per_step"] or 0) * args.steps
                line["kernel_errors"] = res["errors"]
                line["native_library"] = res["lib"]
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
