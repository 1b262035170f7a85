import math

import pytest
import torch

from mia_train_b200.algorithms.dinov3.losses import DINOLoss, IBOTPatchLoss, KoLeoLoss, sinkhorn_knopp
from mia_train_b200.algorithms.dinov3.multicrop import AugmentationConfig, block_mask, photometric, random_resized_crop
from mia_train_b200.algorithms.dinov3_ssl import DINOv3
from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D


def test_sinkhorn_marginals():
    torch.manual_seed(0)
    logits = torch.randn(16, 32)  # (B, K)
    q = sinkhorn_knopp(logits, 0.1, n_iterations=20)
    assert q.shape == (16, 32)
    torch.testing.assert_close(q.sum(dim=1), torch.ones(16), atol=1e-4, rtol=0)  # each sample a distribution
    torch.testing.assert_close(q.sum(dim=0), torch.full((32,), 16 / 32), atol=5e-2, rtol=0)  # balanced prototypes


def test_dino_loss_uniform_is_log_k():
    k = 64
    loss = DINOLoss(k)
    student = torch.zeros(2, 4, k)
    teacher = torch.full((2, 4, k), 1.0 / k)
    assert float(loss(student, teacher)) == pytest.approx(math.log(k), rel=1e-5)
    assert float(loss(student, teacher, ignore_diagonal=True)) == pytest.approx(math.log(k), rel=1e-5)


def test_ibot_masked_loss_is_log_k_for_uniform():
    k = 32
    loss = IBOTPatchLoss(k)
    masks = torch.zeros(2, 8, dtype=torch.bool)
    masks[0, :3] = True
    masks[1, 5:] = True
    n = int(masks.sum())
    student = torch.zeros(n, k)
    teacher = torch.full((n, k), 1.0 / k)
    assert float(loss.forward_masked(student, teacher, masks, n_masked_patches=n)) == pytest.approx(math.log(k), rel=1e-5)


def test_koleo_prefers_spread():
    koleo = KoLeoLoss()
    spread = torch.eye(8)
    clumped = torch.eye(8) + 5.0
    assert float(koleo(spread)) < float(koleo(clumped))


def test_block_mask_ratio_bounds():
    torch.manual_seed(0)
    masks = block_mask((4, 4, 4), 16, (0.1, 0.5), sample_probability=1.0)
    assert masks.shape == (16, 64) and masks.dtype == torch.bool
    frac = masks.float().mean(dim=1)
    assert (frac <= 0.5 + 1e-6).all()
    none = block_mask((4, 4, 4), 8, (0.1, 0.5), sample_probability=0.0)
    assert not none.any()


def test_crops_and_photometric_shapes():
    v = torch.randn(3, 1, 24, 24, 24)
    crop = random_resized_crop(v, (16, 16, 16), (0.3, 1.0))
    assert crop.shape == (3, 1, 16, 16, 16) and torch.isfinite(crop).all()
    out = photometric(crop, AugmentationConfig())
    assert out.shape == crop.shape


def make_algorithm(**kw):
    enc = DinoVisionTransformer3D(img_size=32, patch_size=8, embed_dim=32, depth=2, num_heads=2, n_storage_tokens=2)
    args = dict(input_axes="lcxyz", global_crop_size=32, local_crop_size=16, n_local_crops=2, head_n_prototypes=64,
                head_hidden_dim=32, head_bottleneck_dim=16, total_steps=10, warmup_teacher_temp_steps=4)
    args.update(kw)
    return DINOv3(enc, **args)


def test_initial_loss_near_log_k_and_backward():
    torch.manual_seed(0)
    alg = make_algorithm(koleo_loss_weight=0.0, ibot_loss_weight=0.0)
    out = alg({"img": torch.randn(2, 1, 1, 40, 40, 40)})
    assert float(out["dino_global"]) == pytest.approx(math.log(64), rel=0.05)
    out["loss"].backward()
    assert all(p.grad is None for p in alg.teacher.parameters())


def test_schedules():
    alg = make_algorithm(momentum_teacher=0.9, final_momentum_teacher=1.0, warmup_teacher_temp=0.04, teacher_temp=0.07)
    assert alg.current_teacher_temp(0) == pytest.approx(0.04)
    assert alg.current_teacher_temp(4) == pytest.approx(0.07)
    assert alg.current_teacher_temp(100) == pytest.approx(0.07)
    assert alg.current_momentum(0) == pytest.approx(0.9)
    assert alg.current_momentum(10) == pytest.approx(1.0)
    assert 0.9 < alg.current_momentum(5) < 1.0


def test_ema_runs_from_engine_hook():
    alg = make_algorithm()
    before = [p.detach().clone() for p in alg.teacher.parameters()]
    with torch.no_grad():
        for p in alg.student.parameters():
            p.add_(1.0)
    m = alg.current_momentum()
    alg.after_optimizer_step(1)
    for t0, t, s in zip(before, alg.teacher.parameters(), alg.student.parameters(), strict=True):
        torch.testing.assert_close(t, m * t0 + (1 - m) * s)


def test_step_buffer_counts_and_is_checkpointed():
    alg = make_algorithm()
    alg({"img": torch.randn(2, 1, 1, 40, 40, 40)})
    assert alg.step == 1
    assert "_step" in alg.state_dict()
    alg.validation_step({"img": torch.randn(2, 1, 1, 40, 40, 40)})
    assert alg.step == 1


def test_requires_forward_features():
    from mia_train_b200.models.vit import ViT3D

    with pytest.raises(TypeError, match="forward_features"):
        DINOv3(ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2), input_axes="lcxyz")


def test_step_never_reads_device_values(monkeypatch):
    """After the first step (which reads the checkpointed counter once), a training step makes no
    `.item()` call: schedules use a host copy of the step, masks and masked token indices are built
    on the host. On a GPU each such call would stall the launch queue."""
    torch.manual_seed(0)
    alg = make_algorithm()
    batch = {"img": torch.randn(2, 1, 1, 40, 40, 40)}
    alg(batch)
    calls = []
    real = torch.Tensor.item

    def counting(self):
        calls.append(tuple(self.shape))
        return real(self)

    monkeypatch.setattr(torch.Tensor, "item", counting)
    out = alg(batch)
    out["loss"].backward()
    alg.after_optimizer_step(2)
    monkeypatch.setattr(torch.Tensor, "item", real)
    assert calls == []
    assert alg.step == int(alg._step) == 2


def test_host_step_follows_a_loaded_checkpoint():
    alg = make_algorithm()
    alg({"img": torch.randn(2, 1, 1, 40, 40, 40)})
    assert alg.step == 1
    state = alg.state_dict()
    state["_step"] = torch.tensor(7)
    alg.load_state_dict(state)
    assert alg.step == 7
    assert alg.current_teacher_temp() == pytest.approx(alg.current_teacher_temp(7))
