"""Every shipped run config builds through the registries and trains one step on CPU.

The model, LoRA and algorithm sections are taken as written, except that depth is capped at 2
and, where the objective allows, the crop at 64^3 (CPU time); the data section is built as
written with its crop capped the same way. The workload configs also match the constants the
benchmark modules time, so the two cannot drift apart.
"""

from __future__ import annotations

import dataclasses
from pathlib import Path

import pytest
import torch
from torch.utils.data import default_collate

from mia_train_b200 import components  # noqa: F401
from mia_train_b200.algorithms.registry import AlgorithmRegistry
from mia_train_b200.data.registry import DataRegistry
from mia_train_b200.engine.run import prepare_model
from mia_train_b200.utils.config import load_run_config

CONFIGS = Path(__file__).resolve().parents[2] / "configs"
RUN_CONFIGS = sorted(p for p in CONFIGS.rglob("*.toml") if "cluster" not in p.parts)
CAP = 64


def _capped(config):
    model = dict(config.model.kwargs)
    data = dict(config.data.kwargs)
    model["depth"] = min(int(model.get("depth", 2)), 2)
    if config.algorithm.name != "dinov3":  # its crop sizes fix the volume and model sizes
        size = model.get("img_size")
        if size is not None and (max(size) if isinstance(size, list) else size) > CAP:
            model["img_size"] = CAP if isinstance(size, int) else [CAP] * len(size)
        if "shape" in data:
            data["shape"] = [min(int(v), CAP) for v in data["shape"]]
    return dataclasses.replace(
        config,
        model=dataclasses.replace(config.model, kwargs=model),
        data=dataclasses.replace(config.data, kwargs=data),
    )


def test_every_run_config_is_covered():
    names = {p.relative_to(CONFIGS).as_posix() for p in RUN_CONFIGS}
    assert {"mae_smoke_synthetic.toml", "muvit_mae_smoke_synthetic.toml", "affinity_smoke_synthetic.toml",
            "dinov3_lora_smoke_synthetic.toml", "dinov3_ssl_smoke_synthetic.toml", "semantic_seg_smoke_synthetic.toml",
            "workloads/vit_l_mae.toml", "workloads/dinov3_vit_h.toml",
            "workloads/windowed_simmim_vit_l.toml", "workloads/affinity_vit_l_tp2.toml"} <= names


@pytest.mark.parametrize("path", RUN_CONFIGS, ids=lambda p: p.relative_to(CONFIGS).as_posix())
def test_config_trains_one_step(path):
    config = _capped(load_run_config(path))
    torch.manual_seed(0)
    dataset = DataRegistry.build(config.data.name, **config.data.kwargs)
    model = prepare_model(config)
    algorithm = AlgorithmRegistry.build(config.algorithm.name, model, dataset, **config.algorithm.kwargs)
    transform = algorithm.sample_transform()
    if transform is not None:
        dataset.attach_transform(transform)
    batch = default_collate([dataset.dataset[i] for i in range(min(2, config.trainer.batch_size))])
    algorithm.train()
    out = algorithm.training_step(batch)
    loss = out["loss"]
    assert torch.isfinite(loss.detach())
    loss.backward()
    trainable = [p for p in algorithm.parameters() if p.requires_grad]
    assert trainable and any(p.grad is not None and p.grad.abs().sum() > 0 for p in trainable)


def test_workload_configs_match_benchmarks():
    from mia_train_b200.benchmarks import affinity_tp, dinov3_dp, windowed_tp

    dino = load_run_config(CONFIGS / "workloads" / "dinov3_vit_h.toml")
    for key, value in dinov3_dp.MODEL.items():
        assert dino.model.kwargs[key] == value, key
    for key, value in dinov3_dp.ALG.items():
        got = dino.algorithm.kwargs[key]
        assert (tuple(got) if isinstance(value, tuple) else got) == value, key
    assert dino.trainer.batch_size == dinov3_dp.BATCH and dino.data.kwargs["shape"] == [dinov3_dp.SIDE] * 3

    win = load_run_config(CONFIGS / "workloads" / "windowed_simmim_vit_l.toml")
    for key, value in {**windowed_tp.MODEL, **windowed_tp.WINDOW}.items():
        assert win.model.kwargs[key] == value, key
    assert win.algorithm.kwargs["mask_ratio"] == windowed_tp.MASK_RATIO
    assert win.trainer.activation_checkpointing and win.parallelism.tp == 4

    aff = load_run_config(CONFIGS / "workloads" / "affinity_vit_l_tp2.toml")
    for key, value in affinity_tp.MODEL.items():
        assert aff.model.kwargs[key] == value, key
    assert aff.trainer.batch_size == affinity_tp.BATCH and aff.parallelism.tp == 2
    assert aff.algorithm.kwargs["offsets"] == "nisb12" and aff.algorithm.kwargs["decoder"] == "subpixel"
