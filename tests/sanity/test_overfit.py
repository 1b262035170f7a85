"""Sanity tier: the framework can fit one fixed batch (reference `tests/sanity/test_overfit.py`).

Each test trains through the engine's own optimizer grouping, AdamW and warmup/decay schedule, so
a broken gradient path, a parameter group that never steps or a schedule stuck at zero shows up as
a loss that does not fall.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn as nn
from torch.utils.data import default_collate

from mia_train_b200.algorithms.affinity_seg import AffinitySegmentation
from mia_train_b200.algorithms.mae import MAE
from mia_train_b200.algorithms.semantic_seg import SemanticSegmentation
from mia_train_b200.data.synthetic import SyntheticVolumes
from mia_train_b200.engine.config import TrainerConfig
from mia_train_b200.engine.optimizer import build_lr_scheduler, build_optimizer
from mia_train_b200.models.vit import ViT3D


def _fit(module: nn.Module, loss_fn, steps: int, lr: float) -> tuple[float, float]:
    config = TrainerConfig(max_steps=steps, batch_size=1, lr=lr, warmup_steps=5, weight_decay=0.0,
                           fused_optimizer="off", grad_clip_norm=1.0)
    opt = build_optimizer(module, config)
    schedule = build_lr_scheduler(opt, config)
    losses = []
    for _ in range(steps):
        loss = loss_fn()
        loss.backward()
        opt.step()
        schedule.step()
        opt.zero_grad(set_to_none=True)
        losses.append(float(loss.detach()))
    return losses[0], min(losses[-5:])


def test_mlp_overfits_one_batch():
    torch.manual_seed(0)
    mlp = nn.Sequential(nn.Linear(8, 64), nn.GELU(), nn.Linear(64, 1))
    x, y = torch.randn(16, 8), torch.randn(16, 1)
    first, last = _fit(mlp, lambda: (mlp(x) - y).square().mean(), 200, 1e-2)
    assert last < 0.1 * first


def test_mae_overfits_one_volume():
    torch.manual_seed(0)
    vit = ViT3D(img_size=(16, 16, 16), patch_size=(4, 4, 4), embed_dim=64, depth=2, num_heads=4)
    mae = MAE(vit, input_axes="lcxyz", mask_ratio=0.5, decoder_embed_dim=32, decoder_depth=1, decoder_num_heads=2)
    batch = default_collate([SyntheticVolumes(generator="blobs", shape=(16, 16, 16)).dataset[0]])
    first, last = _fit(mae, lambda: mae.training_step(batch)["loss"], 150, 3e-3)
    assert last < 0.25 * first


@pytest.mark.parametrize("decoder", ["interpolate", "subpixel"])
def test_affinity_overfits_one_volume(decoder):
    torch.manual_seed(0)
    vit = ViT3D(img_size=(16, 16, 16), patch_size=(4, 4, 4), embed_dim=64, depth=2, num_heads=4)
    data = SyntheticVolumes(generator="voronoi", shape=(16, 16, 16), n_seeds=12)
    alg = AffinitySegmentation(vit, data, decoder=decoder, decoder_hidden_dim=16, long_range=3)
    transform = alg.sample_transform()
    if transform is not None:
        data.attach_transform(transform)
    batch = default_collate([data.dataset[0]])
    first, last = _fit(alg, lambda: alg.training_step(batch)["loss"], 150, 3e-3)
    assert last < 0.8 * first


def test_semantic_seg_overfits_one_volume():
    torch.manual_seed(0)
    vit = ViT3D(img_size=(16, 16, 16), patch_size=(4, 4, 4), embed_dim=64, depth=2, num_heads=4)
    data = SyntheticVolumes(generator="voronoi", shape=(16, 16, 16), n_seeds=12, classes=4)
    alg = SemanticSegmentation(vit, data, num_classes=4, decoder_hidden_dim=16)
    batch = default_collate([data.dataset[0]])
    first, last = _fit(alg, lambda: alg.training_step(batch)["loss"], 150, 3e-3)
    assert last < 0.5 * first
