"""Every algorithm's training step on the native kernels (bf16) against the PyTorch-math oracle."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU collection
    pytest.skip("needs CUDA", allow_module_level=True)

from mia_train_b200 import components  # noqa: E402,F401
from mia_train_b200.algorithms.affinity_seg import AffinitySegmentation  # noqa: E402
from mia_train_b200.algorithms.dinov3_ssl import DINOv3  # noqa: E402
from mia_train_b200.algorithms.muvit_mae import MuViTMAE  # noqa: E402
from mia_train_b200.algorithms.semantic_seg import SemanticSegmentation  # noqa: E402
from mia_train_b200.algorithms.simmim import SimMIM  # noqa: E402
from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D  # noqa: E402
from mia_train_b200.models.muvit import MuViT3D  # noqa: E402
from mia_train_b200.models.vit import ViT3D  # noqa: E402
from mia_train_b200.ops import _native  # noqa: E402

DEV = torch.device("cuda", 0)


def run(alg, batch, seed=0):
    """Loss and parameter gradients of one step, native bf16 and reference fp32-math bf16."""
    out = {}
    for mode in ("native", "reference"):
        alg.zero_grad(set_to_none=True)
        torch.manual_seed(seed)
        torch.cuda.manual_seed(seed)
        ctx = _native.reference_math() if mode == "reference" else torch.enable_grad()
        with ctx, torch.autocast("cuda", dtype=torch.bfloat16):
            metrics = alg(batch)
        metrics["loss"].float().backward()
        grads = {n: p.grad.float().clone() for n, p in alg.named_parameters() if p.grad is not None}
        out[mode] = (float(metrics["loss"]), grads)
    assert _native.native().check_errors(0) == 0
    return out


def check(out, loss_tol=3e-2, grad_tol=0.15):
    (ln, gn), (lr, gr) = out["native"], out["reference"]
    assert abs(ln - lr) <= loss_tol * max(1.0, abs(lr)), (ln, lr)
    assert set(gn) == set(gr)
    worst = []
    for name in gr:
        ref = gr[name]
        scale = ref.norm().item() + 1e-6
        err = (gn[name] - ref).norm().item() / scale
        worst.append((err, name))
    worst.sort(reverse=True)
    assert worst[0][0] < grad_tol, worst[:5]


def vit3d():
    return ViT3D(img_size=(32, 32, 32), patch_size=(8, 8, 8), embed_dim=128, depth=2, num_heads=4)


def test_simmim_on_dinov3_windowed_swiglu():
    enc = DinoVisionTransformer3D(img_size=32, patch_size=4, embed_dim=128, depth=2, num_heads=4, n_storage_tokens=4,
                                  ffn_layer="swiglu", layerscale_init=0.1, mask_k_bias=True, window_size=4,
                                  global_every=2).to(DEV)
    alg = SimMIM(enc, input_axes="lcxyz", mask_ratio=0.6, mask_granularity=2).to(DEV)
    batch = {"img": torch.randn(2, 1, 1, 32, 32, 32, device=DEV)}
    check(run(alg, batch))


def test_affinity_subpixel_nisb12():
    alg = AffinitySegmentation(vit3d(), input_axes="lcxyz", decoder="subpixel", offsets="nisb12",
                               decoder_hidden_dim=32, decoder_zero_init_output=False, split_disconnected=False).to(DEV)
    labels = torch.randint(0, 5, (2, 1, 32, 32, 32), device=DEV)
    batch = {"img": torch.randn(2, 1, 1, 32, 32, 32, device=DEV), "label": labels}
    check(run(alg, batch))


def test_semantic_interpolate():
    alg = SemanticSegmentation(vit3d(), input_axes="lcxyz", num_classes=6, decoder_hidden_dim=32).to(DEV)
    batch = {"img": torch.randn(2, 1, 1, 32, 32, 32, device=DEV),
             "label": torch.randint(-1, 6, (2, 1, 32, 32, 32), device=DEV)}
    check(run(alg, batch))


def test_muvit_mae():
    enc = MuViT3D(levels=(1, 2), img_size=(32, 32, 32), patch_size=(8, 8, 8), embed_dim=128, depth=2, num_heads=4)
    alg = MuViTMAE(enc, input_axes="lcxyz", decoder_embed_dim=64, decoder_depth=1, decoder_num_heads=2).to(DEV)
    batch = {"img": torch.randn(2, 2, 1, 32, 32, 32, device=DEV), "bbox": enc.default_bbox(2, DEV)}
    check(run(alg, batch))


def test_dinov3_ssl_step_and_ema():
    enc = DinoVisionTransformer3D(img_size=32, patch_size=8, embed_dim=128, depth=2, num_heads=4, n_storage_tokens=2)
    alg = DINOv3(enc, input_axes="lcxyz", global_crop_size=32, local_crop_size=16, n_local_crops=2,
                 head_n_prototypes=256, head_hidden_dim=128, head_bottleneck_dim=64).to(DEV)
    batch = {"img": torch.randn(2, 1, 1, 40, 40, 40, device=DEV)}
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = alg(batch)
    out["loss"].backward()
    assert torch.isfinite(out["loss"]).item()
    before = [p.detach().clone() for p in alg.teacher.parameters()]
    alg.after_optimizer_step(1)
    moved = any(not torch.equal(a, b) for a, b in zip(before, alg.teacher.parameters(), strict=True))
    assert moved or all(torch.equal(p, q) for p, q in zip(alg.teacher.parameters(), alg.student.parameters()))
    assert _native.native().check_errors(0) == 0


@pytest.mark.parametrize("b,k,iters", [(37, 4096, 3), (3, 65536, 3), (64, 1024, 0), (16, 2048, 1), (300, 8192, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sinkhorn_native_matches_reference(b, k, iters, dtype):
    """Scaling-vector Sinkhorn on native reductions against the reference's matrix iteration."""
    from mia_train_b200.algorithms.dinov3.losses import _sinkhorn_native, sinkhorn_knopp
    from mia_train_b200.ops import _native as _nat

    torch.manual_seed(41)
    logits = (torch.randn(b, k, device="cuda") * 0.3).to(dtype)  # exp(x / T) stays finite, as the reference needs
    got = _sinkhorn_native(logits, 0.07, iters, float(b))
    with _nat.reference_math():
        ref = sinkhorn_knopp(logits, 0.07, iters)
    assert got.shape == ref.shape and got.dtype == torch.float32
    torch.testing.assert_close(got, ref, rtol=1e-3, atol=1e-6 * float(ref.abs().max()))
    torch.testing.assert_close(got.sum(dim=1), ref.sum(dim=1), rtol=1e-4, atol=1e-4)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
@pytest.mark.parametrize("norm_pix", [False, True])
def test_simmim_masked_l1_native(norm_pix):
    from mia_train_b200.ops.mae import masked_l1, masked_l1_reference

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    vol = torch.randn(2, 1, 32, 32, 32, device=dev, generator=g)
    mask = torch.rand(2, 64, device=dev, generator=g) < 0.6
    pred = torch.randn(2, 64, 512, device=dev, generator=g).bfloat16().requires_grad_(True)
    loss, vis = masked_l1(pred, vol, mask, (8, 8, 8), norm_pix)
    loss.backward()
    pr = pred.detach().float().requires_grad_(True)
    rl, rv = masked_l1_reference(pr, vol, mask, (8, 8, 8), norm_pix)
    rl.backward()
    assert abs(float(loss) - float(rl)) < 1e-3 * max(1.0, abs(float(rl)))
    assert abs(float(vis) - float(rv)) < 1e-3 * max(1.0, abs(float(rv)))
    # sign gradients: compare where the reference's |diff| is not tiny (bf16 prediction)
    assert float((pred.grad.float() - pr.grad).abs().max()) <= 2.0 / 512 / float(mask.sum()) + 1e-9
