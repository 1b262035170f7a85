"""Micro-benchmarks of single native ops against their PyTorch/cuBLAS counterparts.

    python -m mia_train_b200.ops.microbench gemm --m 2048 --n 4096 --k 1024 [--layout nt|nn|tn|tt]
    python -m mia_train_b200.ops.microbench mae-step-gemms
    python -m mia_train_b200.ops.microbench attention --b 16 --h 16 --n 512 --d 32

Times are CUDA-event averages after warm-up, with a synchronize on both sides. Layout letters
give A then B: `n` = K-major ("normal" for D = A B^T), `t` = the transposed (M- or N-major) read.
The GEMM shapes of `mae-step-gemms` are the forward and backward GEMMs of one ViT-L MAE step
(per-rank batch 16, 128 visible of 512 tokens).
"""

from __future__ import annotations

import argparse

import torch

from .linear import gemm


def _time(fn, iters: int = 20, warmup: int = 5) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters * 1000.0  # microseconds


def bench_gemm(m: int, n: int, k: int, layout: str = "nn", iters: int = 20, out_fp32: bool = False) -> dict:
    dev = torch.device("cuda")
    a = torch.randn(m, k, device=dev).bfloat16()
    b = torch.randn(n, k, device=dev).bfloat16()
    a_k, b_k = layout[0] == "n", layout[1] == "n"
    a_in = a if a_k else a.t().contiguous()
    b_in = b if b_k else b.t().contiguous()
    out = torch.empty(m, n, device=dev, dtype=torch.float32 if out_fp32 else torch.bfloat16)
    us = _time(lambda: gemm(a_in, b_in, a_kmajor=a_k, b_kmajor=b_k, out=out), iters)
    am = a_in if a_k else a_in.t()
    bm = b_in if b_k else b_in.t()
    us_cublas = _time(lambda: torch.matmul(am, bm.t()), iters)
    flops = 2.0 * m * n * k
    return {
        "shape": (m, n, k),
        "layout": layout,
        "us": us,
        "tflops": flops / us / 1e6,
        "cublas_us": us_cublas,
        "cublas_tflops": flops / us_cublas / 1e6,
    }


# (name, M, N, K, layout, fp32 out) for one ViT-L MAE step: forward, dX (W read N-major), dW.
def mae_step_gemms(batch: int = 16) -> list[tuple[str, int, int, int, str, bool]]:
    enc, dec = batch * 128, batch * 512
    shapes = []
    for tag, m, d, h in (("enc", enc, 1024, 4096), ("dec", dec, 512, 2048)):
        for name, n, k in (("qkv", 3 * d, d), ("proj", d, d), ("fc1", h, d), ("fc2", d, h)):
            shapes.append((f"{tag}.{name}.fwd", m, n, k, "nn", False))
            shapes.append((f"{tag}.{name}.dx", m, k, n, "nt", False))
            shapes.append((f"{tag}.{name}.dw", n, k, m, "tt", True))
    shapes.append(("patch_embed.fwd", enc, 1024, 4096, "nn", False))
    shapes.append(("head.fwd", dec, 4096, 512, "nn", False))
    return shapes


def bench_attention(b: int, h: int, n: int, d: int, iters: int = 20) -> dict:
    from . import _native

    dev = torch.device("cuda")
    q, k, v = (torch.randn(b, h, n, d, device=dev).bfloat16() for _ in range(3))
    o = torch.empty(b, n, h, d, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(b, h, n, device=dev)
    scale = d**-0.5
    ext = _native.native()
    fwd_us = _time(lambda: ext.attention_fwd(q, k, v, o, lse, scale), iters)
    do = torch.randn_like(o)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    bwd_us = _time(lambda: ext.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, scale), iters)
    sdpa_us = _time(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale), iters)
    flops = 4.0 * b * h * n * n * d
    return {"fwd_us": fwd_us, "fwd_tflops": flops / fwd_us / 1e6, "bwd_us": bwd_us,
            "bwd_tflops": 2.5 * flops / bwd_us / 1e6, "sdpa_fwd_us": sdpa_us}


def main() -> None:
    ap = argparse.ArgumentParser(prog="python -m mia_train_b200.ops.microbench")
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=2048)
    g.add_argument("--n", type=int, default=4096)
    g.add_argument("--k", type=int, default=1024)
    g.add_argument("--layout", default="nn")
    g.add_argument("--iters", type=int, default=20)
    g.add_argument("--fp32-out", action="store_true")
    s = sub.add_parser("mae-step-gemms")
    s.add_argument("--batch", type=int, default=16)
    s.add_argument("--iters", type=int, default=20)
    at = sub.add_parser("attention")
    for name, default in (("b", 16), ("h", 16), ("n", 512), ("d", 32), ("iters", 20)):
        at.add_argument(f"--{name}", type=int, default=default)
    args = ap.parse_args()
    if args.cmd == "gemm":
        print(bench_gemm(args.m, args.n, args.k, args.layout, args.iters, args.fp32_out))
    elif args.cmd == "attention":
        print(bench_attention(args.b, args.h, args.n, args.d, args.iters))
    else:
        tot, tot_cb = 0.0, 0.0
        for name, m, n, k, layout, fp32 in mae_step_gemms(args.batch):
            r = bench_gemm(m, n, k, layout, args.iters, fp32)
            tot += r["us"]
            tot_cb += r["cublas_us"]
            print(f"{name:18s} {m:6d} {n:6d} {k:6d} {layout}  native {r['us']:8.1f} us {r['tflops']:7.1f} TF/s"
                  f"   cuBLAS {r['cublas_us']:8.1f} us {r['cublas_tflops']:7.1f} TF/s")
        print(f"total one encoder+decoder block set: native {tot:.1f} us, cuBLAS {tot_cb:.1f} us")


if __name__ == "__main__":
    main()
