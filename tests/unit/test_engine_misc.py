import contextlib
import json
from pathlib import Path

import pytest
import torch
import torch.nn as nn

from mia_train_b200.algorithms.mae import MAE
from mia_train_b200.engine.activation_checkpoint import apply_activation_checkpointing, checkpointable_targets
from mia_train_b200.engine.checkpoint import CheckpointManager
from mia_train_b200.engine.config import LoRAConfig, TrainerConfig
from mia_train_b200.engine.lora import apply_lora
from mia_train_b200.engine.mfu import ThroughputMeter, measure_step_flops
from mia_train_b200.engine.optimizer import build_optimizer
from mia_train_b200.engine.profiler import summarize, union_length
from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
from mia_train_b200.models.vit import ViT3D


def vit():
    return ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=2)


def test_checkpoint_roundtrip_and_latest(tmp_path):
    torch.manual_seed(0)
    m = nn.Linear(4, 4)
    opt = build_optimizer(m, TrainerConfig(max_steps=5, batch_size=1, fused_optimizer="off"))
    m(torch.randn(2, 4)).sum().backward()
    opt.step()
    mgr = CheckpointManager(m, opt, tmp_path)
    mgr.save(3)
    mgr.save(7)
    (tmp_path / "step_9.tmp").mkdir()  # an interrupted save is never "latest"
    assert mgr.available_steps() == [3, 7]
    saved = m.weight.detach().clone()
    with torch.no_grad():
        m.weight.zero_()
    m2 = nn.Linear(4, 4)
    opt2 = build_optimizer(m2, TrainerConfig(max_steps=5, batch_size=1, fused_optimizer="off"))
    step = CheckpointManager(m2, opt2, tmp_path).load_latest()
    assert step == 7
    torch.testing.assert_close(m2.weight, saved)
    assert opt2.state_dict()["state"]
    with pytest.raises(ValueError):
        CheckpointManager(m2, opt2, tmp_path).load_step(5)


def test_resume_with_a_parameter_that_never_had_a_gradient(tmp_path):
    """A trainable parameter no loss has reached yet has no optimizer state in the checkpoint; the
    resume loads everything else and leaves that parameter without state, as it was saved."""

    class TwoHeads(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.used = nn.Linear(4, 4)
            self.unused = nn.Linear(4, 4)  # e.g. a head whose loss term has not fired yet

    def build():
        m = TwoHeads()
        return m, build_optimizer(m, TrainerConfig(max_steps=5, batch_size=1, fused_optimizer="off"))

    torch.manual_seed(0)
    m, opt = build()
    m.used(torch.randn(2, 4)).sum().backward()
    opt.step()
    CheckpointManager(m, opt, tmp_path).save(1)
    m2, opt2 = build()
    assert CheckpointManager(m2, opt2, tmp_path).load_latest() == 1
    torch.testing.assert_close(m2.used.weight, m.used.weight)
    state = opt2.state_dict()["state"]
    saved = opt.state_dict()["state"]
    assert len(state) == len(saved) == 2  # used.weight and used.bias only
    m2.used(torch.randn(2, 4)).sum().backward()
    opt2.step()  # the resumed optimizer steps normally


def test_activation_checkpointing_wraps_declared_blocks():
    alg = MAE(vit(), input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    targets = checkpointable_targets(alg)
    assert len(targets) == 3  # two encoder blocks, one decoder block
    n = apply_activation_checkpointing(alg)
    assert n == 3
    out = alg({"img": torch.randn(2, 1, 1, 16, 16, 16)})
    out["loss"].backward()
    with pytest.raises(ValueError):
        apply_activation_checkpointing(nn.Linear(2, 2))


def test_every_transformer_declares_blocks():
    from mia_train_b200 import components  # noqa: F401
    from mia_train_b200.models.muvit import MuViT3D

    for m in (vit(), DinoVisionTransformer3D(img_size=16, patch_size=8, embed_dim=32, depth=2, num_heads=2),
              MuViT3D(levels=(1, 2), img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=2)):
        assert len(m.checkpointable_modules()) == 2


def test_lora_freezes_base_and_trains_adapters():
    m = vit()
    report = apply_lora(m, LoRAConfig(rank=4, alpha=8.0, targets=("attn_qkv", "mlp")))
    assert report.adapted and report.adapter_params > 0
    trainable = {n for n, p in m.named_parameters() if p.requires_grad}
    assert any("lora_a" in n for n in trainable)
    assert "blocks.0.attn.qkv.weight" not in trainable
    x = torch.randn(1, 1, 16, 16, 16)
    y0 = m(x)
    assert torch.isfinite(y0).all()
    with pytest.raises(ValueError):
        apply_lora(vit(), LoRAConfig(rank=4, alpha=8.0, targets=("nope",)))


@pytest.mark.parametrize("mask_k_bias", [False, True])
def test_lora_adapters_train_on_every_dinov3_target(mask_k_bias):
    """Every adapted layer of a DINOv3 encoder is in the graph (a masked-key-bias qkv included), and
    the adapted forward equals the forward of the merged weights."""
    torch.manual_seed(0)
    m = DinoVisionTransformer3D(img_size=16, patch_size=8, embed_dim=32, depth=2, num_heads=2,
                                qkv_bias=True, mask_k_bias=mask_k_bias)
    apply_lora(m, LoRAConfig(rank=4, alpha=8.0, targets=("attn_qkv", "attn_proj", "mlp")))
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("lora_b"):
                p.normal_(0.0, 0.5)  # a trained adapter: its delta changes the output
    x = torch.randn(2, 1, 16, 16, 16)
    out = m.forward_features(x)["x_norm_patchtokens"]
    out.square().mean().backward()
    adapters = {n: p for n, p in m.named_parameters() if "lora_" in n}
    assert len(adapters) == 2 * 2 * 4  # 2 blocks x (qkv, proj, fc1, fc2) x (A, B)
    for name, p in adapters.items():
        assert p.grad is not None and p.grad.abs().sum() > 0, name
    with torch.no_grad():
        for module in m.modules():
            if hasattr(module, "merge_lora"):
                module.merge_lora()
        torch.testing.assert_close(m.forward_features(x)["x_norm_patchtokens"], out.detach(), atol=1e-5, rtol=1e-4)


def test_flop_counter_sees_attention():
    alg = MAE(vit(), input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    flops = measure_step_flops(alg, {"img": torch.randn(2, 1, 1, 16, 16, 16)}, contextlib.nullcontext)
    assert flops > 0
    assert all(p.grad is None for p in alg.parameters())


def test_throughput_meter_discards_first_window():
    meter = ThroughputMeter(step_flops=int(1e12), peak_flops=2e12, samples_per_step=4)
    meter.start()
    assert meter.window(5) is None
    t = meter.window(5)
    assert t is not None and t.samples_per_s > 0
    m = t.as_metrics()
    assert {"mfu", "tflops_per_s", "samples_per_s"} <= set(m)


def test_profiler_summary_from_synthetic_trace(tmp_path):
    trace = {"traceEvents": [
        {"ph": "X", "cat": "kernel", "name": "k1", "ts": 0, "dur": 100, "pid": 0, "tid": 7},
        {"ph": "X", "cat": "kernel", "name": "k2", "ts": 150, "dur": 50, "pid": 0, "tid": 7},
        {"ph": "X", "cat": "user_annotation", "name": "forward", "ts": 0, "dur": 120, "pid": 1, "tid": 1},
    ]}
    path = tmp_path / "t.pt.trace.json"
    path.write_text(json.dumps(trace))
    text = summarize(path)
    assert "k1" in text and "forward" in text
    assert union_length([(0, 10), (5, 20), (30, 40)]) == 30


def test_raise_on_device_errors_reads_and_reports(monkeypatch):
    from mia_train_b200.ops import _native

    monkeypatch.setattr(_native, "native_available", lambda: True)
    codes = iter([0, 402])
    monkeypatch.setattr(_native, "device_error_code", lambda device: next(codes))
    _native.raise_on_device_errors(0)  # clean word: nothing raised
    with pytest.raises(_native.DeviceWaitError, match="gradient-norm exchange"):
        _native.raise_on_device_errors(0)
    _native.raise_on_device_errors(torch.device("cpu"))  # CPU: never reads a device word
