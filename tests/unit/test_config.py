from pathlib import Path

import pytest

from mia_train_b200.utils.config import diff_resolved, flatten_resolved, load_run_config, parse_run_config

CONFIGS = Path(__file__).resolve().parents[2] / "configs"


def minimal(**extra):
    raw = {
        "experiment_name": "t",
        "model": {"name": "vit3d", "embed_dim": 64},
        "algorithm": {"name": "mae"},
        "data": {"name": "synthetic_volumes"},
        "trainer": {"max_steps": 3, "batch_size": 2},
    }
    raw.update(extra)
    return raw


def test_parse_minimal_and_components():
    cfg = parse_run_config(minimal())
    assert cfg.model.name == "vit3d" and cfg.model.kwargs == {"embed_dim": 64}
    assert cfg.trainer.max_steps == 3
    assert cfg.parallelism.world_size == 1


def test_unknown_keys_rejected():
    with pytest.raises(ValueError, match="unknown key"):
        parse_run_config(minimal(trainer={"max_steps": 1, "batch_size": 1, "bogus": 1}))
    with pytest.raises(ValueError, match="unknown key"):
        parse_run_config(minimal(parallelism={"dp_shard": 1, "pp": 2}))


def test_missing_sections_and_name():
    raw = minimal()
    del raw["data"]
    with pytest.raises(ValueError, match="missing"):
        parse_run_config(raw)
    with pytest.raises(ValueError, match="name"):
        parse_run_config(minimal(model={"embed_dim": 3}))


def test_lora_and_freeze_exclusive():
    with pytest.raises(ValueError, match="LoRA|lora"):
        parse_run_config(minimal(lora={"rank": 4, "targets": ["attn_qkv"]},
                                 trainer={"max_steps": 50, "batch_size": 1, "freeze_backbone_steps": 5}))


def test_shipped_configs_parse():
    paths = sorted(p for p in CONFIGS.rglob("*.toml") if "cluster" not in p.parts)
    assert paths
    for p in paths:
        load_run_config(p)


def test_flatten_and_diff():
    a = {"model": {"kwargs": {"depth": 2, "dim": 8}}, "x": 1}
    b = {"model": {"kwargs": {"depth": 4, "dim": 8}}, "y": 2}
    flat = flatten_resolved(a)
    assert flat["model.kwargs.depth"] == 2
    d = diff_resolved(a, b)
    assert d["model.kwargs.depth"] == (2, 4)
    assert "x" in d and "y" in d and "model.kwargs.dim" not in d
