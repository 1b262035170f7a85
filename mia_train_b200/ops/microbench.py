"""Micro-benchmarks of single native ops against their PyTorch/cuBLAS counterparts.

    python -m mia_train_b200.ops.microbench gemm --m 2048 --n 4096 --k 1024 [--layout nt|nn|tn|tt]
    python -m mia_train_b200.ops.microbench mae-step-gemms
    python -m mia_train_b200.ops.microbench attention --b 16 --h 16 --n 512 --d 32
    python -m mia_train_b200.ops.microbench step-gemms [--depth 24]   # device time of every GEMM of a real step

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


def bench_gemm(m: int, n: int, k: int, layout: str = "nn", iters: int = 20, out_fp32: bool = False,
               act: str = "none") -> dict:
    from .linear import ACT_DGELU, ACT_GELU, ACT_NONE

    dev = torch.device("cuda")
    a = torch.randn(m, k, device=dev).bfloat16()
    b = torch.randn(n, k, device=dev).bfloat16()
    a_k, b_k = layout[0] == "n", layout[1] == "n"
    a_in = a if a_k else a.t().contiguous()
    b_in = b if b_k else b.t().contiguous()
    out = torch.empty(m, n, device=dev, dtype=torch.float32 if out_fp32 else torch.bfloat16)
    code = {"none": ACT_NONE, "gelu": ACT_GELU, "dgelu": ACT_DGELU}[act]
    extra = torch.randn(m, n, device=dev).bfloat16() if act != "none" else None
    kw = {"aux_out": extra} if act == "gelu" else {"aux": extra} if act == "dgelu" else {}
    us = _time(lambda: gemm(a_in, b_in, a_kmajor=a_k, b_kmajor=b_k, out=out, act=code, **kw), iters)
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


def bench_attention(b: int, h: int, n: int, d: int, iters: int = 20, tc_mode: int = 1, poly: int = 1) -> dict:
    """Native attention forward / backward on (b, h, n, d) bf16; tc_mode 1 = tcgen05 kernels where
    they apply, 0 = warp-level kernels. FLOPs: 4 b h n^2 d forward, 2.5x that backward."""
    from . import _native

    dev = torch.device("cuda")
    ext = _native.native()
    previous = ext.tc_attention_mode()
    ext.set_tc_attention_mode(tc_mode)
    previous_poly = ext.set_attention_poly_exp(poly)
    try:
        q, k, v = (torch.randn(b, h, n, d, device=dev).bfloat16() for _ in range(3))
        o = torch.empty(b, n, h, d, device=dev, dtype=torch.bfloat16)
        lse = torch.empty(b, h, n, device=dev)
        scale = d**-0.5
        fwd_us = _time(lambda: ext.attention_fwd(q, k, v, o, lse, scale), iters)
        do = torch.randn_like(o)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        bwd_us = _time(lambda: ext.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, scale), iters)
        sdpa_us = _time(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale), iters)
        # SDPA backward alone: one forward with autograd, then time the backward of that graph
        qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
        out_g = torch.nn.functional.scaled_dot_product_attention(qg, kg, vg, scale=scale)
        go = torch.randn_like(out_g)
        sdpa_bwd_us = _time(lambda: torch.autograd.grad(out_g, (qg, kg, vg), go, retain_graph=True), iters)
    finally:
        ext.set_tc_attention_mode(previous)
        ext.set_attention_poly_exp(previous_poly)
    flops = 4.0 * b * h * n * n * d
    return {"tc_mode": tc_mode, "poly_exp": poly, "shape": [b, h, n, d], "fwd_us": round(fwd_us, 2), "fwd_tflops": round(flops / fwd_us / 1e6, 1),
            "bwd_us": round(bwd_us, 2), "bwd_tflops": round(2.5 * flops / bwd_us / 1e6, 1),
            "sdpa_fwd_us": round(sdpa_us, 2), "sdpa_bwd_us": round(sdpa_bwd_us, 2),
            "fwd_vs_sdpa": round(sdpa_us / fwd_us, 3), "bwd_vs_sdpa": round(sdpa_bwd_us / bwd_us, 3)}


def bench_sinkhorn(b: int, k: int, iters: int = 3, reps: int = 20) -> dict:
    """Sinkhorn-Knopp centring of (b, k) fp32 teacher logits: native scaling-vector kernels against
    the matrix iteration in PyTorch ops (`reference_math`)."""
    from ..algorithms.dinov3.losses import sinkhorn_knopp
    from . import _native

    logits = torch.randn(b, k, device="cuda") * 0.3
    native_us = _time(lambda: sinkhorn_knopp(logits, 0.07, iters), reps)
    with _native.reference_math():
        torch_us = _time(lambda: sinkhorn_knopp(logits, 0.07, iters), reps)
    return {"shape": (b, k), "iterations": iters, "native_us": round(native_us, 1), "torch_us": round(torch_us, 1)}


def step_gemms(depth: int = 24, batch: int = 16) -> str:
    """Device time of each GEMM launched by one eager ViT-L MAE training step, grouped by shape."""
    from collections import defaultdict

    from torch.profiler import ProfilerActivity, profile

    from ..algorithms.mae import MAE
    from ..models.vit import ViT3D
    from . import linear

    dev = torch.device("cuda")
    torch.manual_seed(0)
    model = ViT3D(img_size=(128,) * 3, patch_size=(16,) * 3, embed_dim=1024, depth=depth, num_heads=16, mlp_ratio=4.0)
    alg = MAE(model, input_axes="lcxyz", mask_ratio=0.75, decoder_embed_dim=512, decoder_depth=8,
              decoder_num_heads=16).to(dev)
    x = torch.randn(batch, 1, 1, 128, 128, 128, device=dev)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = alg({"img": x})
        out["loss"].backward()
        alg.zero_grad(set_to_none=True)

    step()
    torch.cuda.synchronize()
    linear.GEMM_TRACE = []
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    trace, linear.GEMM_TRACE = linear.GEMM_TRACE, None
    kernels = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
                      and "gemm_tcgen05" in e.name), key=lambda e: e.time_range.start)
    if len(kernels) != len(trace):
        return f"unmatched: {len(kernels)} GEMM kernels vs {len(trace)} calls"
    agg: dict[tuple, list[float]] = defaultdict(lambda: [0.0, 0, 0.0])
    for call, kern in zip(trace, kernels, strict=True):
        us = kern.device_time_total
        m, n, k = call[:3]
        key = (*call, "pair" if "pair" in kern.name else "single", kern.name.split("<")[1].split(",")[0])
        agg[key][0] += us
        agg[key][1] += 1
        agg[key][2] += 2.0 * m * n * k
    total = sum(v[0] for v in agg.values())
    flops = sum(v[2] for v in agg.values())
    lines = [f"GEMMs of one step: {total / 1000:.3f} ms device time, {flops / 1e12:.3f} TFLOP, "
             f"{flops / total / 1e6:.1f} TF/s average"]
    for key, (us, cnt, f) in sorted(agg.items(), key=lambda kv: -kv[1][0]):
        m, n, k, layout, dt, act, accum, res, kind, bn = key
        lines.append(f"  {m:6d} {n:6d} {k:6d} {layout} {dt:4s} act={act} acc={int(accum)} res={int(res)} {kind:6s} BN={bn:3s}"
                     f"  x{cnt:3d}  {us / cnt:8.1f} us  {f / us / 1e6:7.1f} TF/s  ({100 * us / total:4.1f}%)")
    return "\n".join(lines)


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
    g.add_argument("--act", choices=("none", "gelu", "dgelu"), default="none")
    s = sub.add_parser("mae-step-gemms")
    s.add_argument("--batch", type=int, default=16)
    s.add_argument("--iters", type=int, default=20)
    s.add_argument("--pair-modes", default="0,2",
                   help="GEMM tile modes to compare (0 = single-CTA tiles, 2 = CTA pairs when M >= 256)")
    sg = sub.add_parser("step-gemms")
    sg.add_argument("--depth", type=int, default=24)
    sg.add_argument("--batch", type=int, default=16)
    at = sub.add_parser("attention")
    for name, default in (("b", 16), ("h", 16), ("n", 512), ("d", 32), ("iters", 20)):
        at.add_argument(f"--{name}", type=int, default=default)
    at.add_argument("--modes", default="1,0", help="attention kernels: 1 = tcgen05, 0 = warp-level mma")
    at.add_argument("--poly", default="1", help="comma list: 1 = a quarter of the exponentials on the FMA pipe, 0 = none")
    sk = sub.add_parser("sinkhorn")
    sk.add_argument("--b", type=int, default=2048)
    sk.add_argument("--k", type=int, default=65536)
    sk.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    if args.cmd == "sinkhorn":
        print(bench_sinkhorn(args.b, args.k, args.iters))
        return
    if args.cmd == "step-gemms":
        print(step_gemms(args.depth, args.batch))
        return
    if args.cmd == "gemm":
        print(bench_gemm(args.m, args.n, args.k, args.layout, args.iters, args.fp32_out, args.act))
    elif args.cmd == "attention":
        for mode in (int(x) for x in args.modes.split(",")):
            for poly in (int(x) for x in args.poly.split(",")):
                print(bench_attention(args.b, args.h, args.n, args.d, args.iters, mode, poly))
    else:
        from . import _native

        modes = [int(x) for x in args.pair_modes.split(",")]
        totals = dict.fromkeys(modes, 0.0)
        tot_cb = 0.0
        for name, m, n, k, layout, fp32 in mae_step_gemms(args.batch):
            cols = []
            for mode in modes:
                previous = _native.native().set_gemm_pair_mode(mode)
                r = bench_gemm(m, n, k, layout, args.iters, fp32)
                _native.native().set_gemm_pair_mode(previous)
                totals[mode] += r["us"]
                cols.append(f"mode{mode} {r['us']:7.1f} us {r['tflops']:6.1f} TF/s")
            tot_cb += r["cublas_us"]
            print(f"{name:18s} {m:6d} {n:6d} {k:6d} {layout}  " + "  ".join(cols)
                  + f"   cuBLAS {r['cublas_us']:7.1f} us {r['cublas_tflops']:6.1f} TF/s")
        print("total one encoder+decoder block set: " + ", ".join(f"mode{m} {t:.1f} us" for m, t in totals.items())
              + f", cuBLAS {tot_cb:.1f} us")


if __name__ == "__main__":
    main()
