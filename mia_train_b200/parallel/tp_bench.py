"""Microbenchmark of the sequence-parallel TP collective GEMMs: fused kernels vs NCCL + GEMM.

    torchrun --nnodes=1 --nproc-per-node W --master-addr 127.0.0.1 --master-port P \\
        -m mia_train_b200.parallel.tp_bench [--tokens 32768] [--dim 1024] [--iters 20]

For the four GEMMs of a ViT block at `tokens` tokens and width `dim` over a TP group of W GPUs
(qkv and fc1: all-gather -> GEMM; proj and fc2: GEMM -> reduce-scatter, with bias and residual),
rank 0 prints one JSON line per op with the device time (CUDA events around each launch, L2
flushed before it, ranks aligned by a barrier, max over ranks and median over iterations) of the
fused kernel and of the collective baseline (NCCL all-gather / reduce-scatter around the same
native GEMM), and the fused kernel's fraction of its roofline: the slower of its FLOPs at the
measured bf16 GEMM peak and its NVLink bytes (what this rank must receive or send) at the measured
peer bandwidth per direction.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics

import torch
import torch.distributed as dist

PEAK_FLOPS = 1410.2e12  # measured sustained cuBLAS bf16 on this pool's B200s
LINK_BPS = 770e9  # measured peer copy bandwidth per direction per GPU


AG_POINTS = ("start", "first-N-tile slices stored", "first block pushed", "all blocks pushed",
             "producer reached peers' tiles", "MMA done", "epilogue done", "exit")
RS_POINTS = ("start", "MMA done", "epilogue done", "peer tiles landed", "first own block's partials present", "-",
             "-", "exit")


def _timeline(trace: torch.Tensor, kind: int) -> dict:
    """{point: [min, median, max] us after the earliest CTA start} over the CTAs that recorded it in
    this launch (a CTA's entries are kept from its own start on)."""
    t = trace[kind]
    t = t[t[:, 0] > 0]
    if t.numel() == 0:
        return {}
    t0 = int(t[:, 0].min())
    names = AG_POINTS if kind == 0 else RS_POINTS
    out = {}
    for i, name in enumerate(names):
        col = t[:, i]
        col = col[col >= t[:, 0]]
        if name == "-" or col.numel() == 0:
            continue
        us = (col - t0).double() / 1000.0
        out[name] = [round(float(us.min()), 1), round(float(us.median()), 1), round(float(us.max()), 1)]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--dim", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    from ..ops import _native
    from ..ops.linear import ACT_GELU, gemm
    from ..ops.tp import TpComm, ag_gemm, gemm_rs

    m = -(-args.tokens // (world * 128)) * world * 128 if args.tokens % world else args.tokens
    s = m // world
    c = args.dim
    g = torch.Generator(device=dev).manual_seed(rank)
    fused = TpComm(dist.group.WORLD, "fused")
    coll = TpComm(dist.group.WORLD, "collective")
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)

    def rnd(*shape):
        return (torch.randn(*shape, device=dev, generator=g) * 0.05).bfloat16()

    x_r = rnd(s, c)
    w_qkv, w_fc1 = rnd(3 * c // world, c), rnd(4 * c // world, c)
    w_proj, w_fc2 = rnd(c, c // world), rnd(c, 4 * c // world)
    b_qkv, b_fc1, b_c = (torch.randn(n, device=dev, generator=g) for n in (3 * c // world, 4 * c // world, c))
    o_full, u_full = rnd(m, c // world), rnd(m, 4 * c // world)
    res = rnd(s, c)

    ops = {
        "qkv all-gather->GEMM": (lambda cm: ag_gemm(cm, x_r, w_qkv, bias=b_qkv), 2 * m * c * 3 * c // world,
                                 (world - 1) * s * c * 2),
        "fc1 all-gather->GEMM+GELU": (lambda cm: ag_gemm(cm, x_r, w_fc1, bias=b_fc1, act=ACT_GELU, want_pre=True),
                                      2 * m * c * 4 * c // world, (world - 1) * s * c * 2),
        "proj GEMM->reduce-scatter+residual": (lambda cm: gemm_rs(cm, o_full, w_proj, bias=b_c, residual=res),
                                               2 * m * (c // world) * c, (world - 1) * s * c * 2),
        "fc2 GEMM->reduce-scatter+residual": (lambda cm: gemm_rs(cm, u_full, w_fc2, bias=b_c, residual=res),
                                              2 * m * (4 * c // world) * c, (world - 1) * s * c * 2),
    }
    del gemm
    results = []
    for name, (fn, flops, link_bytes) in ops.items():
        times = {}
        for label, cm in (("fused", fused), ("nccl", coll)):
            samples = []
            for it in range(args.warmup + args.iters):
                flush.zero_()
                dist.barrier()
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn(cm)
                b.record()
                torch.cuda.synchronize()
                if it >= args.warmup:
                    samples.append(a.elapsed_time(b))
            t = torch.tensor([statistics.median(samples)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times[label] = float(t) * 1e-3
        # the fused result against the collective one (same GEMM kernel, NCCL transfer)
        outs = [fn(cm) for cm in (fused, coll)]
        outs = [o[0] if isinstance(o, tuple) else o for o in outs]
        rel = torch.tensor([float((outs[0].float() - outs[1].float()).norm() / (outs[1].float().norm() + 1e-12))],
                           device=dev)
        dist.all_reduce(rel, op=dist.ReduceOp.MAX)
        roof = max(flops / PEAK_FLOPS, link_bytes / LINK_BPS)
        results.append({"op": name, "tokens": m, "dim": c, "tp": world, "fused_us": round(times["fused"] * 1e6, 1),
                        "nccl_us": round(times["nccl"] * 1e6, 1), "speedup": round(times["nccl"] / times["fused"], 3),
                        "roofline_us": round(roof * 1e6, 1), "fused_frac_of_roofline": round(roof / times["fused"], 3),
                        "tflops": round(flops / times["fused"] / 1e12, 1),
                        "link_gbs": round(link_bytes / times["fused"] / 1e9, 1),
                        "rel_err_vs_nccl": round(float(rel), 5)})
    traces = {}
    if os.environ.get("MIA_TP_TRACE") == "1":
        # one more launch of each fused op, then its per-CTA timeline (us after the first CTA started)
        for name, (fn, _, _) in ops.items():
            dist.barrier()
            torch.cuda.synchronize()
            fn(fused)
            torch.cuda.synchronize()
            traces[name] = _timeline(_native.native().tp_trace_read(local), 0 if "all-gather" in name else 1)
    errors = int(_native.native().check_errors(local))
    if rank == 0:
        for r in results:
            print(json.dumps({**r, "kernel_errors": errors}), flush=True)
        for name, tl in traces.items():
            print(json.dumps({"trace": name, "rank": rank, "points_us": tl}), flush=True)
    dist.barrier()
    fused.release()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
