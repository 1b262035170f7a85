"""The benchmark workload modules behind `bench.py --config`: each exposes the same contract, and
the analytic FLOP counts that feed the MFU column have the expected magnitude."""

from __future__ import annotations

import importlib
import importlib.util
from pathlib import Path

import pytest
import torch

CONFIGS = ("windowed_tp", "affinity_tp", "dinov3_dp")


@pytest.mark.parametrize("name", CONFIGS)
def test_module_contract(name):
    mod = importlib.import_module(f"mia_train_b200.benchmarks.{name}")
    for attr in ("METRIC", "DATA", "SEQ_LEN", "describe", "native_arm", "reference_arm"):
        assert hasattr(mod, attr), f"{name} lacks {attr}"
    assert "samples/sec" in mod.METRIC and "synthetic" in mod.DATA
    d = mod.describe(8)
    assert isinstance(d, dict) and "model" in d


def test_bench_lists_every_config():
    spec = importlib.util.spec_from_file_location("bench_under_test", Path(__file__).resolve().parents[2] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert set(bench.EXTRA_CONFIGS) == set(CONFIGS)


def test_dinov3_step_flops_magnitude():
    from mia_train_b200.benchmarks import dinov3_dp
    from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D

    with torch.device("meta"):
        m = DinoVisionTransformer3D(**dinov3_dp.MODEL)
    n_params = sum(p.numel() for p in m.parameters())
    assert 6.0e8 < n_params < 7.0e8  # ViT-H class
    # 2 * params * tokens per pass: teacher 16 global crops, student 16 global + 64 local, backward 2x
    tokens_teacher = dinov3_dp.BATCH * 2 * 517
    tokens_student = dinov3_dp.BATCH * (2 * 517 + 8 * 69)
    rough = 2 * n_params * (tokens_teacher + 3 * tokens_student)
    f = dinov3_dp._step_flops(m)
    assert 0.9 * rough < f < 1.4 * rough
