"""Numerics of every native kernel against a plain fp32 PyTorch version of the same op.

Run on a B200: `python -m pytest tests -m gpu`. Each test also checks that no kernel recorded a
bounded-wait timeout in the device error word.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU, skipped there
    pytest.skip("needs CUDA", allow_module_level=True)

from mia_train_b200.ops import _native  # noqa: E402
from mia_train_b200.ops.linear import ACT_DGELU, ACT_GELU, gelu_grad_reference, gemm  # noqa: E402

DEV = torch.device("cuda", 0)


def _no_errors():
    torch.cuda.synchronize()
    assert _native.native().check_errors(0) == 0


def _close(actual, expected, rel=2e-2, atol=2e-2):
    a, e = actual.float(), expected.float()
    err = (a - e).abs().max().item()
    scale = e.abs().max().item() + 1e-6
    assert err <= atol + rel * scale, f"max error {err:.4g} vs scale {scale:.4g}"


@pytest.fixture(params=[0, 2], ids=["single_cta", "cta_pairs"])
def pair_mode(request):
    from mia_train_b200.ops._native import native

    previous = native().set_gemm_pair_mode(request.param)
    yield request.param
    native().set_gemm_pair_mode(previous)


@pytest.mark.parametrize("a_k,b_k", [(True, True), (True, False), (False, True), (False, False)])
@pytest.mark.parametrize("mnk", [(256, 256, 128), (384, 648, 200), (128, 136, 64), (2048, 3072, 1024), (1000, 512, 4096),
                                 (640, 200, 64)])
def test_gemm_layouts(a_k, b_k, mnk, pair_mode):
    m, n, k = mnk
    torch.manual_seed(0)
    a = torch.randn(m, k, device=DEV).bfloat16()
    b = torch.randn(n, k, device=DEV).bfloat16()
    ref = a.float() @ b.float().t()
    a_in = a if a_k else a.t().contiguous()
    b_in = b if b_k else b.t().contiguous()
    out = gemm(a_in, b_in, a_kmajor=a_k, b_kmajor=b_k, out_dtype=torch.float32)
    _close(out, ref, rel=1e-2, atol=1e-2 * math.sqrt(k))
    _no_errors()


@pytest.mark.parametrize("b_k", [True, False])
def test_gemm_ragged_rows(b_k, pair_mode):
    """M not a multiple of 8 (token counts like B * (prefix + patches)), K-major A."""
    m, n, k = 1034, 384, 264
    torch.manual_seed(2)
    a = torch.randn(m, k, device=DEV).bfloat16()
    b = torch.randn(n, k, device=DEV).bfloat16()
    bias = torch.randn(n, device=DEV)
    out = gemm(a, b if b_k else b.t().contiguous(), b_kmajor=b_k, bias=bias, out_dtype=torch.float32)
    _close(out, a.float() @ b.float().t() + bias, rel=1e-2, atol=1e-2 * math.sqrt(k))
    # weight-gradient form: the 1034 tokens are the K dimension, both operands read M/N-major
    dy = torch.randn(m, n, device=DEV).bfloat16()
    dw = gemm(dy, a, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32)
    _close(dw, dy.float().t() @ a.float(), rel=1e-2, atol=1e-2 * math.sqrt(m))
    _no_errors()


def test_gemm_epilogues(pair_mode):
    torch.manual_seed(1)
    m, n, k = 512, 768, 320
    a = torch.randn(m, k, device=DEV).bfloat16()
    b = (torch.randn(n, k, device=DEV) * 0.05).bfloat16()
    bias = torch.randn(n, device=DEV)
    gamma = torch.rand(n, device=DEV)
    res = torch.randn(m, n, device=DEV).bfloat16()
    acc = a.float() @ b.float().t() + bias
    pre = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    y = gemm(a, b, bias=bias, act=ACT_GELU, aux_out=pre)
    _close(pre, acc, rel=1e-2, atol=5e-2)
    _close(y, F.gelu(acc), rel=1e-2, atol=5e-2)
    y2 = gemm(a, b, bias=bias, gamma=gamma, residual=res)
    _close(y2, res.float() + gamma * acc, rel=1e-2, atol=5e-2)
    y3 = gemm(a, b, act=ACT_DGELU, aux=res)
    _close(y3, (a.float() @ b.float().t()) * gelu_grad_reference(res.float()), rel=1e-2, atol=5e-2)
    out = torch.randn(m, n, device=DEV)
    base = out.clone()
    gemm(a, b, out=out, accumulate=True)
    _close(out, base + a.float() @ b.float().t(), rel=1e-2, atol=5e-2)
    _no_errors()


def test_gelu_epilogue_matches_exact_erf_gelu():
    """fp32 GELU / GELU' epilogues against torch's exact-erf GELU on exactly representable inputs."""
    torch.manual_seed(3)
    m, n, k = 256, 512, 64
    # small integers / 8: every product and sum is exact in fp32, so the pre-activation is exact
    a = (torch.randint(-8, 9, (m, k), device=DEV).float() / 8).bfloat16()
    b = (torch.randint(-8, 9, (n, k), device=DEV).float() / 64).bfloat16()
    pre = a.float() @ b.float().t()
    y = gemm(a, b, act=ACT_GELU, out_dtype=torch.float32)
    torch.testing.assert_close(y, F.gelu(pre), atol=3e-6, rtol=1e-6)
    aux = pre.bfloat16()
    g = gemm(a, b, act=ACT_DGELU, aux=aux, out_dtype=torch.float32)
    torch.testing.assert_close(g, pre * gelu_grad_reference(aux.float()), atol=3e-6, rtol=2e-6)
    _no_errors()


@pytest.mark.parametrize("m,n", [(3000, 520), (8192, 512), (7, 64), (2048, 4096), (130, 1032), (65, 8)])
def test_column_sum(m, n):
    from mia_train_b200.ops.linear import column_sum

    x = torch.randn(m, n, device=DEV).bfloat16()
    _close(column_sum(x), x.float().sum(0), rel=1e-3, atol=1e-2)
    acc = torch.ones(n, device=DEV)
    column_sum(x, out=acc, accumulate=True)
    _close(acc, x.float().sum(0) + 1.0, rel=1e-3, atol=1e-2)
    _no_errors()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rms", [False, True])
def test_layernorm(dtype, rms):
    from mia_train_b200.ops.norm import layer_norm, rms_norm

    torch.manual_seed(2)
    x = (torch.randn(777, 1024, device=DEV) * 3 + 1).to(dtype).requires_grad_(True)
    w = torch.randn(1024, device=DEV, requires_grad=True)
    b = torch.randn(1024, device=DEV, requires_grad=True)
    dy = torch.randn(777, 1024, device=DEV).to(dtype)
    if rms:
        y = rms_norm(x, w, 1e-6)
        xf = x.detach().float().requires_grad_(True)
        wf = w.detach().clone().requires_grad_(True)
        ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
        params, ref_params = (w,), (wf,)
    else:
        y = layer_norm(x, w, b, 1e-5)
        xf = x.detach().float().requires_grad_(True)
        wf = w.detach().clone().requires_grad_(True)
        bf = b.detach().clone().requires_grad_(True)
        ref = F.layer_norm(xf, (1024,), wf, bf, 1e-5)
        params, ref_params = (w, b), (wf, bf)
    _close(y, ref)
    y.backward(dy)
    ref.backward(dy.float())
    _close(x.grad, xf.grad, rel=2e-2, atol=5e-2)
    for p, rp in zip(params, ref_params, strict=True):
        _close(p.grad, rp.grad, rel=1e-2, atol=1e-1)
    _no_errors()


@pytest.mark.parametrize("shape", [(2, 4, 128, 64), (2, 3, 200, 32), (1, 2, 512, 32), (1, 2, 96, 128)])
def test_attention_fwd_bwd(shape):
    from mia_train_b200.ops.attention import attention

    torch.manual_seed(3)
    b, h, n, d = shape
    q = torch.randn(b, n, h, d, device=DEV).bfloat16().requires_grad_(True)
    k = torch.randn(b, n, h, d, device=DEV).bfloat16().requires_grad_(True)
    v = torch.randn(b, n, h, d, device=DEV).bfloat16().requires_grad_(True)
    scale = d**-0.5
    out = attention(q, k, v, scale)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2), scale=scale).transpose(1, 2)
    _close(out, ref)
    dout = torch.randn_like(out)
    out.backward(dout)
    ref.backward(dout.float())
    for g, rg in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        _close(g, rg, rel=3e-2, atol=3e-2)
    _no_errors()


@pytest.mark.parametrize("b,n,h,d", [(2, 128, 4, 64), (3, 77, 2, 32), (1, 200, 3, 128)])
def test_rope_attention_matches_reference(b, n, h, d):
    from mia_train_b200.layers.common.rope import AxialRotaryEmbedding
    from mia_train_b200.ops import attention as attn_ops

    torch.manual_seed(4)
    rot = AxialRotaryEmbedding(d, 3).to(DEV)
    coords = torch.randint(0, 8, (b, n, 3), device=DEV).float()
    qkv = torch.randn(b, n, 3, h, d, device=DEV).bfloat16().requires_grad_(True)
    tables = rot(coords)
    out = attn_ops.rope_attention(qkv, tables.angles, tables.pairs, d**-0.5)
    dout = torch.randn_like(out)
    out.backward(dout)
    g_native = qkv.grad.clone()
    f_native = [f.grad.clone() for f in rot.inv_freqs]
    qkv.grad = None
    for f in rot.inv_freqs:
        f.grad = None
    with _native.reference_math():
        qkv32 = qkv.detach().float().requires_grad_(True)
        tables = rot(coords)
        ref = attn_ops.rope_attention(qkv32, tables.angles, tables.pairs, d**-0.5)
        ref.backward(dout.float())
    _close(out, ref)
    _close(g_native, qkv32.grad, rel=3e-2, atol=3e-2)
    for fn, f in zip(f_native, rot.inv_freqs, strict=True):
        _close(fn, f.grad, rel=5e-2, atol=5e-2)
    _no_errors()


def test_axial_angles_native_matches_torch():
    from mia_train_b200.layers.common.rope import AxialRotaryEmbedding

    torch.manual_seed(8)
    rot = AxialRotaryEmbedding(64, 3).to(DEV)
    coords = torch.randn(4, 37, 3, device=DEV) * 10
    ang = rot.angles(coords)
    g = torch.randn_like(ang)
    ang.backward(g)
    got = [f.grad.clone() for f in rot.inv_freqs]
    for f in rot.inv_freqs:
        f.grad = None
    with _native.reference_math():
        ref = rot.angles(coords)
        ref.backward(g)
    torch.testing.assert_close(ang, ref, atol=1e-5, rtol=1e-6)
    for a, f in zip(got, rot.inv_freqs, strict=True):
        torch.testing.assert_close(a, f.grad, atol=1e-2, rtol=1e-4)
    _no_errors()


@pytest.mark.parametrize("b,n,h,d", [(2, 128, 4, 64), (2, 100, 2, 32)])
def test_packed_attention_without_rope(b, n, h, d):
    from mia_train_b200.ops import attention as attn_ops

    torch.manual_seed(6)
    qkv = torch.randn(b, n, 3, h, d, device=DEV).bfloat16().requires_grad_(True)
    out = attn_ops.rope_attention(qkv, None, None, d**-0.5)
    dout = torch.randn_like(out)
    out.backward(dout)
    with _native.reference_math():
        qkv32 = qkv.detach().float().requires_grad_(True)
        ref = attn_ops.rope_attention(qkv32, None, None, d**-0.5)
        ref.backward(dout.float())
    _close(out, ref)
    _close(qkv.grad, qkv32.grad, rel=3e-2, atol=3e-2)
    _no_errors()


def test_dinov3_rope_attention_shared_angles():
    """DINOv3 layout: prefix tokens unrotated, pairs (i, i + D/2), angles shared by the batch."""
    from mia_train_b200.layers.dinov3.attention import half_pairs
    from mia_train_b200.ops import attention as attn_ops

    torch.manual_seed(7)
    b, n, h, d = 3, 69, 4, 64
    pairs = half_pairs(d, DEV)
    ang = torch.randn(1, n, d // 2, device=DEV).requires_grad_(True)
    with torch.no_grad():
        ang[:, :5] = 0.0
    qkv = torch.randn(b, n, 3, h, d, device=DEV).bfloat16().requires_grad_(True)
    out = attn_ops.rope_attention(qkv, ang, pairs, d**-0.5)
    dout = torch.randn_like(out)
    out.backward(dout)
    g_ang = ang.grad.clone()
    ang.grad = None
    with _native.reference_math():
        qkv32 = qkv.detach().float().requires_grad_(True)
        ref = attn_ops.rope_attention(qkv32, ang, pairs, d**-0.5)
        ref.backward(dout.float())
    _close(out, ref)
    _close(qkv.grad, qkv32.grad, rel=3e-2, atol=3e-2)
    _close(g_ang, ang.grad, rel=5e-2, atol=5e-2)
    _no_errors()


def test_fused_adamw_matches_torch():
    from mia_train_b200.engine.fused_adamw import FusedAdamW

    torch.manual_seed(5)
    shapes = [(300, 70), (1000,), (64, 64, 3), (5,)]
    params = [torch.randn(s, device=DEV, requires_grad=True) for s in shapes]
    ref_params = [p.detach().clone().requires_grad_(True) for p in params]
    groups = [{"params": params[:2], "weight_decay": 0.1}, {"params": params[2:], "weight_decay": 0.0, "lr": 3e-3}]
    ref_groups = [{"params": ref_params[:2], "weight_decay": 0.1}, {"params": ref_params[2:], "weight_decay": 0.0, "lr": 3e-3}]
    opt = FusedAdamW(groups, lr=1e-3, betas=(0.9, 0.95))
    ref = torch.optim.AdamW(ref_groups, lr=1e-3, betas=(0.9, 0.95))
    for _ in range(5):
        for p, rp in zip(params, ref_params, strict=True):
            g = torch.randn_like(p)
            p.grad = g.clone()
            rp.grad = g.clone()
        opt.step()
        ref.step()
    for p, rp in zip(params, ref_params, strict=True):
        torch.testing.assert_close(p, rp, rtol=1e-5, atol=1e-6)
    assert float(opt.state[params[0]]["step"]) == 5.0
    _no_errors()


def test_clip_grad_norm_native():
    from mia_train_b200.ops.optim import clip_grad_norm_native

    params = [torch.nn.Parameter(torch.randn(s, device=DEV)) for s in [(100, 10), (7,), (33, 33)]]
    for p in params:
        p.grad = torch.randn_like(p) * 3
    expected = [p.grad.clone() for p in params]
    total = torch.sqrt(sum((g**2).sum() for g in expected))
    coef = min(1.0, 1.0 / (total.item() + 1e-6))
    norm = clip_grad_norm_native(params, 1.0)
    assert abs(norm.item() - total.item()) < 1e-3 * total.item()
    for p, e in zip(params, expected, strict=True):
        torch.testing.assert_close(p.grad, e * coef, rtol=1e-5, atol=1e-6)
    _no_errors()


def test_mae_ops():
    from mia_train_b200.ops import mae as mae_ops
    from mia_train_b200.ops.patch import patchify, patchify_reference

    torch.manual_seed(6)
    vol = torch.randn(2, 1, 32, 32, 32, device=DEV)
    idx = torch.argsort(torch.rand(2, 64, device=DEV), dim=1)[:, :16]
    rows = patchify(vol, (8, 8, 8), idx, out_dtype=torch.bfloat16)
    ref_rows = torch.gather(patchify_reference(vol, (8, 8, 8)), 1, idx.unsqueeze(-1).expand(-1, -1, 512))
    _close(rows, ref_rows, rel=1e-2, atol=1e-2)
    vis = torch.randn(2, 16, 64, device=DEV).bfloat16().requires_grad_(True)
    tok = torch.randn(1, 1, 64, device=DEV, requires_grad=True)
    restore = torch.argsort(torch.rand(2, 64, device=DEV), dim=1)
    out = mae_ops.restore_with_mask_token(vis, tok, restore)
    ref = mae_ops.restore_reference(vis.detach().float(), tok.detach(), restore)
    _close(out, ref)
    g = torch.randn_like(out)
    out.backward(g)
    vis32 = vis.detach().float().requires_grad_(True)
    tok32 = tok.detach().clone().requires_grad_(True)
    mae_ops.restore_reference(vis32, tok32, restore).backward(g.float())
    _close(vis.grad, vis32.grad)
    _close(tok.grad, tok32.grad, rel=1e-2, atol=1e-1)
    pred = torch.randn(2, 64, 512, device=DEV).bfloat16().requires_grad_(True)
    mask = (torch.rand(2, 64, device=DEV) < 0.75).float()
    loss = mae_ops.norm_pix_mse(pred, vol, mask, (8, 8, 8))
    loss.backward()
    pred32 = pred.detach().float().requires_grad_(True)
    ref_loss = mae_ops.norm_pix_mse_reference(pred32, vol, mask, (8, 8, 8))
    ref_loss.backward()
    assert abs(loss.item() - ref_loss.item()) < 1e-3 * max(1.0, ref_loss.item())
    _close(pred.grad, pred32.grad, rel=2e-2, atol=1e-5)
    _no_errors()


def test_mae_step_native_vs_reference_math():
    """One vit3d+MAE training step: native kernels vs PyTorch math on the same weights and batch."""
    import copy

    from mia_train_b200.algorithms.mae import MAE
    from mia_train_b200.models.vit import ViT3D

    torch.manual_seed(7)
    model = ViT3D(img_size=(32, 32, 32), patch_size=(8, 8, 8), embed_dim=128, depth=2, num_heads=2)
    alg = MAE(model, input_axes="lcxyz", decoder_embed_dim=64, decoder_depth=1, decoder_num_heads=2).to(DEV)
    alg_ref = copy.deepcopy(alg)
    batch = {"img": torch.randn(2, 1, 1, 32, 32, 32, device=DEV)}
    torch.manual_seed(8)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = alg(batch)
    out["loss"].backward()
    torch.manual_seed(8)
    with _native.reference_math(), torch.autocast("cuda", dtype=torch.bfloat16):
        out_ref = alg_ref(batch)
    out_ref["loss"].backward()
    assert abs(out["loss"].item() - out_ref["loss"].item()) < 2e-2 * abs(out_ref["loss"].item())
    for (name, p), (_, pr) in zip(alg.named_parameters(), alg_ref.named_parameters(), strict=True):
        assert p.grad is not None, name
        _close(p.grad, pr.grad, rel=1e-1, atol=1e-3)
    _no_errors()


@pytest.mark.parametrize("mnk", [(512, 512, 8192), (1536, 512, 8192), (1024, 1024, 2048)])
def test_gemm_split_k_weight_gradient(mnk, pair_mode):
    """dW-shaped GEMMs (small output, long K, fp32 accumulate) take the split-K path."""
    m, n, k = mnk
    torch.manual_seed(9)
    dy = torch.randn(k, m, device=DEV).bfloat16()  # (tokens, out) -> A read M-major
    x = torch.randn(k, n, device=DEV).bfloat16()   # (tokens, in)  -> B read N-major
    out = torch.randn(m, n, device=DEV)
    base = out.clone()
    gemm(dy, x, a_kmajor=False, b_kmajor=False, out=out, accumulate=True)
    _close(out, base + dy.float().t() @ x.float(), rel=1e-2, atol=1e-2 * math.sqrt(k))
    fresh = gemm(dy, x, a_kmajor=False, b_kmajor=False, out_dtype=torch.float32)
    _close(fresh, dy.float().t() @ x.float(), rel=1e-2, atol=1e-2 * math.sqrt(k))
    _no_errors()


@pytest.fixture(params=[0, 1], ids=["warp_mma", "tcgen05"])
def tc_attention(request):
    from mia_train_b200.ops._native import native

    previous = native().tc_attention_mode()
    native().set_tc_attention_mode(request.param)
    yield request.param
    native().set_tc_attention_mode(previous)


@pytest.mark.parametrize(
    "b,nq,nk,h,d",
    [(2, 128, 128, 4, 64), (1, 1, 1, 2, 64), (2, 77, 200, 3, 32), (1, 513, 513, 2, 32), (2, 300, 1000, 2, 64),
     (16, 128, 128, 16, 64)],
)
def test_attention_forward_paths(b, nq, nk, h, d, tc_attention):
    """Both forward kernels against fp32 SDPA, incl. ragged query / key tails and a key count
    that is not a multiple of the key block; the tcgen05 path must actually launch."""
    from mia_train_b200.ops._native import native

    torch.manual_seed(11)
    q = torch.randn(b, h, nq, d, device=DEV).bfloat16()
    k = torch.randn(b, h, nk, d, device=DEV).bfloat16()
    v = torch.randn(b, h, nk, d, device=DEV).bfloat16()
    o = torch.empty(b, nq, h, d, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(b, h, nq, device=DEV)
    before = native().tc_attention_launches()
    native().attention_fwd(q, k, v, o, lse, d**-0.5)
    torch.cuda.synchronize()
    assert native().tc_attention_launches() - before == tc_attention
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=d**-0.5)
    _close(o, ref.transpose(1, 2))
    s = (q.float() @ k.float().transpose(-1, -2)) * d**-0.5
    ref_lse = torch.logsumexp(s, dim=-1) / math.log(2.0)
    torch.testing.assert_close(lse, ref_lse, atol=2e-2, rtol=1e-3)
    _no_errors()


@pytest.mark.parametrize("b,n,h,d", [(2, 128, 16, 64), (2, 512, 16, 32), (3, 70, 4, 64)])
def test_attention_packed_views(b, n, h, d, tc_attention):
    """Strided q / k / v straight out of a packed (B, N, 3, H, D) projection, forward and backward."""
    from mia_train_b200.ops import attention as attn_ops

    torch.manual_seed(12)
    qkv = torch.randn(b, n, 3, h, d, device=DEV).bfloat16().requires_grad_(True)
    out = attn_ops.rope_attention(qkv, None, None, d**-0.5)
    dout = torch.randn_like(out)
    out.backward(dout)
    qkv32 = qkv.detach().float().requires_grad_(True)
    q, k, v = (qkv32[:, :, i].transpose(1, 2) for i in range(3))
    ref = F.scaled_dot_product_attention(q, k, v, scale=d**-0.5).transpose(1, 2)
    ref.reshape(out.shape).backward(dout.float())
    _close(out.reshape(ref.shape), ref)
    _close(qkv.grad, qkv32.grad, rel=3e-2, atol=3e-2)
    _no_errors()


@pytest.mark.parametrize(
    "b,nq,nk,h,d", [(2, 128, 128, 4, 64), (2, 77, 200, 3, 32), (1, 513, 513, 2, 32), (2, 300, 260, 2, 64), (1, 1, 1, 1, 64)]
)
def test_attention_backward_paths(b, nq, nk, h, d, tc_attention):
    """Both backward kernels (dq, dk, dv) against fp32 autograd through SDPA, ragged tails incl."""
    from mia_train_b200.ops._native import native

    torch.manual_seed(13)
    q = torch.randn(b, h, nq, d, device=DEV).bfloat16()
    k = torch.randn(b, h, nk, d, device=DEV).bfloat16()
    v = torch.randn(b, h, nk, d, device=DEV).bfloat16()
    o = torch.empty(b, nq, h, d, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(b, h, nq, device=DEV)
    native().attention_fwd(q, k, v, o, lse, d**-0.5)
    dout = torch.randn(b, nq, h, d, device=DEV).bfloat16()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    before = native().tc_attention_launches()
    native().attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, d**-0.5)
    torch.cuda.synchronize()
    assert native().tc_attention_launches() - before == tc_attention
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qf, kf, vf, scale=d**-0.5)
    ref.backward(dout.float().transpose(1, 2))
    for g, rg in ((dq, qf.grad), (dk, kf.grad), (dv, vf.grad)):
        _close(g, rg, rel=3e-2, atol=3e-2)
    _no_errors()


@pytest.mark.parametrize("width", [512, 1024, 1280])
def test_layer_norm_residual_fuses_both_gradients(width):
    """(LN(x), x) with the residual gradient added inside the LayerNorm backward kernel, against
    fp32 autograd of LN(x) and x used separately (weight / bias gradients included)."""
    from mia_train_b200.ops.norm import layer_norm_residual

    torch.manual_seed(21)
    x = (torch.randn(333, width, device=DEV) * 2).bfloat16().requires_grad_(True)
    w = torch.randn(width, device=DEV, requires_grad=True)
    b = torch.randn(width, device=DEV, requires_grad=True)
    dh, dr = torch.randn(333, width, device=DEV).bfloat16(), torch.randn(333, width, device=DEV).bfloat16()
    h, r = layer_norm_residual(x, w, b, 1e-5)
    torch.autograd.backward((h, r), (dh, dr))
    xf = x.detach().float().requires_grad_(True)
    wf, bf = w.detach().clone().requires_grad_(True), b.detach().clone().requires_grad_(True)
    hf = F.layer_norm(xf, (width,), wf, bf, 1e-5)
    torch.autograd.backward((hf, xf * 1.0), (dh.float(), dr.float()))
    _close(h, hf)
    _close(x.grad, xf.grad, rel=2e-2, atol=5e-2)
    _close(w.grad, wf.grad, rel=1e-2, atol=1e-1)
    _close(b.grad, bf.grad, rel=1e-2, atol=1e-1)
    _no_errors()


@pytest.mark.parametrize("shape", [(4, 1, 1, 32, 32, 32), (3, 2, 16, 16, 16), (1, 7, 9, 5)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_zscore_u8(shape, dtype):
    """Native per-volume z-score of uint8 volumes against the float64 torch formula."""
    from mia_train_b200.ops.data import zscore_u8, zscore_u8_reference

    torch.manual_seed(31)
    x = torch.randint(0, 256, shape, dtype=torch.uint8, device=DEV)
    x[0].fill_(7)  # a constant volume: std clamps to 1e-6 -> zeros
    got = zscore_u8(x, dtype)
    ref = zscore_u8_reference(x, torch.float64)
    assert got.dtype == dtype
    _close(got, ref, rel=1e-2 if dtype == torch.bfloat16 else 1e-5, atol=1e-2 if dtype == torch.bfloat16 else 1e-5)
    _no_errors()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
@pytest.mark.parametrize("activation", [None, "gelu"])
def test_lora_linear_native(activation):
    """LoRA delta accumulated into the base GEMM's tile vs the fp32 composition, forward and backward."""
    from mia_train_b200.ops.linear import lora_linear

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    m, k, n, r = 1000, 512, 768, 16
    x = torch.randn(m, k, device=dev, generator=g).bfloat16().requires_grad_(True)
    w = (torch.randn(n, k, device=dev, generator=g) / k**0.5).requires_grad_(True)
    b = torch.randn(n, device=dev, generator=g).requires_grad_(True)
    la = (torch.randn(r, k, device=dev, generator=g) / k**0.5).requires_grad_(True)
    lb = torch.randn(n, r, device=dev, generator=g).requires_grad_(True)
    s = 0.5
    y = lora_linear(x, w, b, la, lb, s, activation=activation)
    assert y is not None
    gy = torch.randn_like(y.float())
    (y.float() * gy).sum().backward()
    xr, wr, br, lar, lbr = (t.detach().float().requires_grad_(True) for t in (x, w, b, la, lb))
    z = xr @ wr.t() + br + s * (xr @ lar.t()) @ lbr.t()
    yr = torch.nn.functional.gelu(z) if activation == "gelu" else z
    (yr * gy).sum().backward()

    def rel(u, v):
        return float((u.float() - v.float()).norm() / (v.float().norm() + 1e-6))

    assert rel(y, yr) < 2e-2
    for got, ref in ((x.grad, xr.grad), (w.grad, wr.grad), (b.grad, br.grad), (la.grad, lar.grad), (lb.grad, lbr.grad)):
        assert rel(got, ref) < 3e-2
