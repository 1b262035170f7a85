"""Native DINO / iBOT soft-target cross-entropy and KoLeo against the fp32 PyTorch formulas."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@needs_cuda
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ignore_diagonal", [False, True])
def test_dino_loss_native(dtype, ignore_diagonal):
    from mia_train_b200.algorithms.dinov3.losses import DINOLoss

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    n_s, n_t, b, k = 4, 2, 3, 4096
    s32 = torch.randn(n_s, b, k, device=dev, generator=g) * 3
    t = torch.softmax(torch.randn(n_t, b, k, device=dev, generator=g) * 4, dim=-1)
    loss_fn = DINOLoss(k, student_temp=0.1)
    s_nat = s32.to(dtype).requires_grad_(True)
    out = loss_fn(s_nat, t, ignore_diagonal=ignore_diagonal)
    out.backward()
    s_ref = s_nat.detach().float().requires_grad_(True)
    logp = F.log_softmax(s_ref / 0.1, dim=-1)
    pair = -torch.einsum("sbk,tbk->st", logp, t)
    if ignore_diagonal:
        pair = pair * (1 - torch.eye(n_s, n_t, device=dev))
        ref = pair.sum() / (b * n_s * n_t - b * min(n_s, n_t))
    else:
        ref = pair.sum() / (b * n_s * n_t)
    ref.backward()
    assert abs(float(out) - float(ref)) < 1e-3 * max(1.0, abs(float(ref)))
    assert _rel(s_nat.grad, s_ref.grad) < (2e-2 if dtype == torch.bfloat16 else 1e-4)


@needs_cuda
def test_ibot_loss_native():
    from mia_train_b200.algorithms.dinov3.losses import IBOTPatchLoss

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    masks = torch.rand(4, 64, device=dev, generator=g) < 0.3
    n = int(masks.sum())
    k = 8192
    s = (torch.randn(n + 5, k, device=dev, generator=g) * 2).bfloat16().requires_grad_(True)
    t = torch.softmax(torch.randn(n + 5, k, device=dev, generator=g) * 3, dim=-1)
    loss_fn = IBOTPatchLoss(k, student_temp=0.1)
    out = loss_fn.forward_masked(s, t, masks, n_masked_patches=n)
    out.backward()
    s_ref = s.detach().float().requires_grad_(True)
    w = (1 / masks.sum(-1).clamp(min=1.0)).unsqueeze(-1).expand_as(masks)[masks]
    per = torch.sum(t * F.log_softmax(s_ref / 0.1, dim=-1), dim=-1)[:n]
    ref = -(per * w).sum() / masks.shape[0]
    ref.backward()
    assert abs(float(out) - float(ref)) < 1e-3 * max(1.0, abs(float(ref)))
    assert _rel(s.grad, s_ref.grad) < 2e-2
    assert float(s.grad[n:].float().abs().max()) == 0.0  # rows past n_masked_patches get no gradient


@needs_cuda
@pytest.mark.parametrize("b,d", [(8, 1280), (33, 256)])
def test_koleo_native(b, d):
    from mia_train_b200.ops.dino import koleo, koleo_reference

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(b)
    x = torch.randn(b, d, device=dev, generator=g)
    xa = x.clone().requires_grad_(True)
    out = koleo(xa)
    out.backward()
    xr = x.clone().requires_grad_(True)
    ref = koleo_reference(xr)
    ref.backward()
    assert abs(float(out) - float(ref)) < 1e-4 * max(1.0, abs(float(ref)))
    assert _rel(xa.grad, xr.grad) < 1e-3


@needs_cuda
def test_prototype_gemm_sinkhorn_colsum():
    """The prototype GEMM's epilogue column sums equal sum_b exp(logits / T), and Sinkhorn fed with
    them equals Sinkhorn computing them itself."""
    from mia_train_b200.algorithms.dinov3.losses import sinkhorn_knopp
    from mia_train_b200.layers.dinov3.head import DINOHead

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    head = DINOHead(in_dim=256, out_dim=8192, nlayers=2, hidden_dim=512, bottleneck_dim=128).to(dev)
    x = torch.randn(200, 256, device=dev)
    temp = 0.07
    colsum = torch.zeros(8192, device=dev)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused = head(x, colsum, temp)
        plain = head(x)
    assert _rel(fused, plain) < 2e-2
    ref = torch.exp(fused.float() / temp).sum(0)
    assert _rel(colsum, ref) < 1e-3
    a = sinkhorn_knopp(fused, temp, 3, colsum=colsum)
    b = sinkhorn_knopp(fused, temp, 3)
    assert _rel(a, b) < 1e-3
