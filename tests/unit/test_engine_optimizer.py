import math

import pytest
import torch
import torch.nn as nn

from mia_train_b200.engine.config import TrainerConfig
from mia_train_b200.engine.optimizer import (
    build_lr_scheduler,
    build_optimizer,
    build_param_groups,
    clip_grad_norm_,
    lr_multiplier,
    weight_decay_at,
)
from mia_train_b200.models.vit import ViT3D


def tiny():
    return ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=3, num_heads=2)


def test_groups_partition_all_trainable_params():
    m = tiny()
    groups = build_param_groups(m, TrainerConfig(max_steps=10, batch_size=1, layerwise_lr_decay=0.8))
    seen = [p for g in groups for p in g["params"]]
    assert len(seen) == len({id(p) for p in seen}) == sum(1 for p in m.parameters() if p.requires_grad)


def test_no_weight_decay_on_vectors():
    m = tiny()
    groups = build_param_groups(m, TrainerConfig(max_steps=10, batch_size=1, weight_decay=0.1))
    for g in groups:
        for p in g["params"]:
            if p.ndim < 2:
                assert g["weight_decay"] == 0.0


def test_layer_decay_orders_blocks():
    m = tiny()
    groups = build_param_groups(m, TrainerConfig(max_steps=10, batch_size=1, layerwise_lr_decay=0.5))
    by_param = {id(p): g["lr_multiplier"] for g in groups for p in g["params"]}
    first = by_param[id(m.blocks[0].attn.qkv.weight)]
    last = by_param[id(m.blocks[2].attn.qkv.weight)]
    assert first < last


@pytest.mark.parametrize("schedule", ["cosine", "linear"])
def test_warmup_then_decay(schedule):
    cfg = TrainerConfig(max_steps=100, batch_size=1, warmup_steps=10, lr_schedule=schedule, min_lr_ratio=0.1)
    vals = [lr_multiplier(s, cfg) for s in range(101)]
    assert vals[0] < vals[5] < vals[10]
    assert vals[10] == pytest.approx(1.0, abs=1e-6)
    assert vals[100] == pytest.approx(0.1, abs=1e-6)
    assert all(a >= b - 1e-12 for a, b in zip(vals[10:], vals[11:]))


def test_scheduler_drives_optimizer_lr():
    m = nn.Linear(4, 4)
    cfg = TrainerConfig(max_steps=20, batch_size=1, lr=1e-3, warmup_steps=5, fused_optimizer="off")
    opt = build_optimizer(m, cfg)
    sched = build_lr_scheduler(opt, cfg)
    lrs = []
    for _ in range(20):
        opt.step()
        sched.step()
        lrs.append(opt.param_groups[0]["lr"])
    assert max(lrs) == pytest.approx(1e-3, rel=1e-6)


def test_weight_decay_schedule_endpoints():
    cfg = TrainerConfig(max_steps=100, batch_size=1, weight_decay=0.04, final_weight_decay=0.2)
    assert weight_decay_at(0, cfg) == pytest.approx(0.04)
    assert weight_decay_at(100, cfg) == pytest.approx(0.2)
    mid = weight_decay_at(50, cfg)
    assert 0.04 < mid < 0.2 and not math.isnan(mid)


def test_clip_grad_norm_matches_torch():
    a = [torch.randn(10, requires_grad=True), torch.randn(3, 4, requires_grad=True)]
    b = [t.detach().clone().requires_grad_(True) for t in a]
    for t, u in zip(a, b):
        g = torch.randn_like(t) * 5
        t.grad = g.clone()
        u.grad = g.clone()
    n1 = clip_grad_norm_(a, 1.0)
    n2 = torch.nn.utils.clip_grad_norm_(b, 1.0)
    torch.testing.assert_close(n1, n2)
    for t, u in zip(a, b):
        torch.testing.assert_close(t.grad, u.grad)
