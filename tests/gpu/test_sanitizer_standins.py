"""Stand-ins for a memory sanitizer on a pool where compute-sanitizer is closed.

* Canaries: outputs are written into the middle of a larger buffer whose guard rows hold a bit
  pattern no kernel produces; after the launch the guards must be bit-for-bit unchanged (an
  out-of-bounds store of any kernel tested here would overwrite them).
* Reruns: kernels without atomics must give bit-identical results on a second run; those that
  accumulate with floating-point atomics (split-K GEMM, the attention dQ accumulator) must agree to
  rounding.
Ragged sizes (rows not a multiple of the tile, the last key block partial) are used throughout,
since that is where an index error would land.
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
GUARD = 3  # guard rows before and after each output
PATTERN = 0x7FA5  # a bf16 NaN payload: no kernel writes it


def _guarded(rows: int, cols: int, dtype=torch.bfloat16, dev="cuda"):
    buf = torch.empty(rows + 2 * GUARD, cols, device=dev, dtype=dtype)
    if dtype == torch.bfloat16:
        buf.view(torch.int16).fill_(PATTERN)
    else:
        buf.view(torch.int32).fill_(0x7FA5A5A5)
    return buf, buf[GUARD:GUARD + rows]


def _guards_intact(buf):
    view = buf.view(torch.int16) if buf.dtype == torch.bfloat16 else buf.view(torch.int32)
    want = PATTERN if buf.dtype == torch.bfloat16 else 0x7FA5A5A5
    return bool((view[:GUARD] == want).all() and (view[-GUARD:] == want).all())


@needs_cuda
@pytest.mark.parametrize("m,n,k", [(1000, 776, 520), (257, 1024, 64), (4096, 136, 1000)])
def test_gemm_canaries_and_rerun(m, n, k):
    from mia_train_b200.ops.linear import ACT_GELU, gemm

    g = torch.Generator(device="cuda").manual_seed(m + n)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        buf, out = _guarded(m, n)
        pbuf, pre = _guarded(m, n)
        gemm(a, w, out=out, bias=bias, act=ACT_GELU, aux_out=pre)
        torch.cuda.synchronize()
        assert _guards_intact(buf) and _guards_intact(pbuf)
        outs.append(out.clone())
    assert torch.equal(outs[0], outs[1])


@needs_cuda
def test_split_k_weight_gradient_rerun():
    """The fp32 split-K path (tokens as K, atomics into the output) agrees with itself to rounding."""
    from mia_train_b200.ops.linear import gemm

    g = torch.Generator(device="cuda").manual_seed(9)
    dy = torch.randn(8192, 256, device="cuda", generator=g).bfloat16()
    x = torch.randn(8192, 384, device="cuda", generator=g).bfloat16()
    runs = []
    for _ in range(2):
        buf, out = _guarded(256, 384, torch.float32)
        gemm(dy, x, a_kmajor=False, b_kmajor=False, out=out)
        torch.cuda.synchronize()
        assert _guards_intact(buf)
        runs.append(out.clone())
    ref = dy.float().t() @ x.float()
    assert float((runs[0] - runs[1]).abs().max()) <= 1e-4 * float(ref.abs().max())
    assert float((runs[0] - ref).norm() / ref.norm()) < 1e-3


@needs_cuda
def test_layer_norm_canaries_and_rerun():
    from mia_train_b200.ops.norm import layer_norm

    x = torch.randn(1003, 1024, device="cuda").bfloat16()
    w, b = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    outs = []
    for _ in range(2):
        y = layer_norm(x, w, b)
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    ref = torch.nn.functional.layer_norm(x.float(), (1024,), w, b)
    assert float((outs[0].float() - ref).abs().max()) < 0.05


@needs_cuda
@pytest.mark.parametrize("n,d", [(577, 64), (200, 32)])
def test_attention_rerun(n, d):
    from mia_train_b200.ops import _native

    ext = _native.native()
    b, h = 2, 4
    g = torch.Generator(device="cuda").manual_seed(n)
    q, k, v = (torch.randn(b, h, n, d, device="cuda", generator=g).bfloat16() for _ in range(3))
    do = torch.randn(b, n, h, d, device="cuda", generator=g).bfloat16()
    scale = 1 / math.sqrt(d)
    res = []
    for _ in range(2):
        # output written between guard batches: o is (B, N, H, D); pad along the batch axis
        ob = torch.empty(b + 2, n, h, d, device="cuda", dtype=torch.bfloat16)
        ob.view(torch.int16).fill_(PATTERN)
        o = ob[1:b + 1]
        lse = torch.empty(b, h, n, device="cuda")
        ext.attention_fwd(q, k, v, o, lse, scale)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ext.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, scale)
        torch.cuda.synchronize()
        raw = ob.view(torch.int16)
        assert bool((raw[0] == PATTERN).all() and (raw[-1] == PATTERN).all())
        res.append((o.clone(), dq.clone(), dk.clone(), dv.clone()))
    assert torch.equal(res[0][0], res[1][0])  # forward: no atomics
    assert torch.equal(res[0][2], res[1][2]) and torch.equal(res[0][3], res[1][3])  # dK, dV per key block
    dq0, dq1 = res[0][1].float(), res[1][1].float()
    assert float((dq0 - dq1).abs().max()) <= 2e-2 * float(dq0.abs().max())  # dQ: fp32 atomics, then bf16
    assert _native.native().check_errors(0) == 0


@needs_cuda
def test_tp_kernels_canaries(tmp_path):
    """The fused TP kernels (one rank) leave the rows around their outputs untouched."""
    import torch.distributed as dist

    from mia_train_b200.ops.tp import TpComm

    created = not dist.is_initialized()
    if created:
        dist.init_process_group("gloo", init_method=f"file://{tmp_path / 'pg'}", rank=0, world_size=1)
    try:
        comm = TpComm(dist.group.WORLD, "fused")
        g = torch.Generator(device="cuda").manual_seed(4)
        x = torch.randn(1000, 256, device="cuda", generator=g).bfloat16()
        w = torch.randn(768, 256, device="cuda", generator=g).bfloat16()
        ws = comm.workspace_for(1000, 768, x.device)
        obuf, out = _guarded(1000, 768)
        fbuf, full = _guarded(1000, 256)
        ws.ag_gemm(x, w, out, full, None, None, None, True, 0)
        rbuf, red = _guarded(1000, 256)
        ws.gemm_rs(out, w, red, None, None, None, None, False)
        torch.cuda.synchronize()
        assert _guards_intact(obuf) and _guards_intact(fbuf) and _guards_intact(rbuf)
        assert torch.equal(full, x)
        comm.release()
    finally:
        if created:
            dist.destroy_process_group()
