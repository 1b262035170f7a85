"""The Trainer's CUDA-graph step mode on one GPU: trains, checkpoints and resumes like eager mode."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU collection
    pytest.skip("needs CUDA", allow_module_level=True)

from mia_train_b200 import components  # noqa: E402,F401
from mia_train_b200.algorithms.mae import MAE  # noqa: E402
from mia_train_b200.data.synthetic import SyntheticVolumes  # noqa: E402
from mia_train_b200.engine.config import TrainerConfig  # noqa: E402
from mia_train_b200.engine.trainer import Trainer  # noqa: E402
from mia_train_b200.models.vit import ViT3D  # noqa: E402


def make_trainer(tmp_path, steps: int, mode: str) -> Trainer:
    torch.manual_seed(0)
    data = SyntheticVolumes(shape=(32, 32, 32), samples_per_epoch=64, generator="blobs", blob_rate=5.0)
    model = ViT3D(img_size=(32, 32, 32), patch_size=(8, 8, 8), embed_dim=128, depth=2, num_heads=4)
    alg = MAE(model, data, decoder_embed_dim=64, decoder_depth=1, decoder_num_heads=4)
    cfg = TrainerConfig(max_steps=steps, batch_size=4, lr=1e-3, warmup_steps=2, precision="bf16", log_every=2,
                        checkpoint_every=4, step_mode=mode, fused_optimizer="on", measure_mfu=False)
    return Trainer(alg, data, cfg, tmp_path, device=torch.device("cuda", 0))


def test_graph_mode_trains_and_resumes(tmp_path):
    trainer = make_trainer(tmp_path, 8, "graph")
    losses = []
    original = trainer.logger.log

    def spy(step, metrics, prefix="train"):
        if prefix == "train":
            losses.append(metrics["loss"])
        return original(step, metrics, prefix=prefix)

    trainer.logger.log = spy
    assert trainer.train() == 8
    assert all(math.isfinite(v) for v in losses) and losses[-1] < losses[0]
    resumed = make_trainer(tmp_path, 10, "graph")
    assert resumed.train() == 10
    eager = make_trainer(tmp_path / "eager", 4, "eager")
    assert eager.train() == 4
