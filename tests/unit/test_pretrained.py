import pytest
import torch
import torch.nn as nn

from mia_train_b200.utils.pretrained import inflate_2d_to_3d, load_pretrained, merge_lora_tensors, read_state_dict


class Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.conv = nn.Conv3d(1, 4, kernel_size=2, stride=2)
        self.fc = nn.Linear(4, 3)


def test_inflate_preserves_response_to_constant_depth():
    w2 = torch.randn(4, 1, 2, 2)
    w3 = inflate_2d_to_3d(w2, torch.Size((4, 1, 2, 2, 2)))
    assert w3.shape == (4, 1, 2, 2, 2)
    torch.testing.assert_close(w3.sum(dim=2), w2, atol=1e-6, rtol=1e-5)


def test_prefix_unwrap_and_strict(tmp_path):
    src = Tiny()
    path = tmp_path / "ck.pth"
    torch.save({"model": {f"backbone.{k}": v for k, v in src.state_dict().items()}}, path)
    dst = Tiny()
    report = load_pretrained(dst, path, prefix="backbone.")
    assert sorted(report.copied) == sorted(src.state_dict())
    torch.testing.assert_close(dst.fc.weight, src.fc.weight)
    with pytest.raises(ValueError):
        load_pretrained(Tiny(), path)  # no prefix: nothing matches


def test_skip_and_unused(tmp_path):
    src = Tiny()
    sd = dict(src.state_dict())
    sd["extra.weight"] = torch.zeros(1)
    path = tmp_path / "ck.pth"
    torch.save(sd, path)
    with pytest.raises(ValueError, match="no home"):
        load_pretrained(Tiny(), path)
    report = load_pretrained(Tiny(), path, allow_unused=True, skip=("fc.",))
    assert report.unused == ["extra.weight"] and "fc.weight" in report.skipped


def test_merge_lora_tensors():
    base = torch.randn(6, 4)
    a = torch.randn(2, 4)
    b = torch.randn(6, 2)
    ck = {"l.weight": base, "l.lora_a": a, "l.lora_b": b, "l.lora_scaling": torch.tensor(0.5)}
    merged, names = merge_lora_tensors(ck)
    assert names
    torch.testing.assert_close(merged["l.weight"], base + 0.5 * b @ a)
    assert not any("lora" in k for k in merged)


def test_read_state_dict_unwraps_teacher(tmp_path):
    path = tmp_path / "t.pth"
    torch.save({"teacher": {"w": torch.ones(1)}}, path)
    assert "w" in read_state_dict(path)


def test_released_2d_dinov3_checkpoint_initialises_the_3d_encoder(tmp_path):
    """The chain the fine-tuning recipes use: a 2-D DINOv3 checkpoint (RGB patch kernel, LayerScale,
    masked key bias, 4 registers) loads strictly into `dinov3_vit3d` through a config's `[init]`
    (inflate_2d_to_3d, rope buffers skipped), and the inflated kernel answers a z-constant volume
    like the 2-D kernel answers its plane."""
    from mia_train_b200 import components  # noqa: F401
    from mia_train_b200.engine.run import prepare_model
    from mia_train_b200.models.dinov3_vit import DinoVisionTransformer
    from mia_train_b200.utils.config import parse_run_config

    torch.manual_seed(0)
    dims = dict(patch_size=8, embed_dim=48, depth=2, num_heads=2, n_storage_tokens=4,
                layerscale_init=1e-5, mask_k_bias=True)
    src = DinoVisionTransformer(img_size=32, in_chans=3, **dims)
    path = tmp_path / "dinov3_2d.pth"
    torch.save(src.state_dict(), path)
    config = parse_run_config({
        "experiment_name": "init_chain",
        "model": {"name": "dinov3_vit3d", "img_size": 32, "in_chans": 1, "pos_embed_rope_type": "superposition",
                  **dims},
        "init": {"path": str(path), "inflate_2d_to_3d": True, "skip": ["rope_embed."], "strict": True},
        "algorithm": {"name": "simmim"},
        "data": {"name": "synthetic_volumes"},
        "trainer": {"max_steps": 1, "batch_size": 1},
    })
    model = prepare_model(config)
    torch.testing.assert_close(model.blocks[1].attn.qkv.weight, src.blocks[1].attn.qkv.weight)
    torch.testing.assert_close(model.blocks[0].ls1.gamma, src.blocks[0].ls1.gamma)
    torch.testing.assert_close(model.storage_tokens, src.storage_tokens)
    # a z-constant single-channel volume through the inflated kernel == the plane through the RGB kernel
    # averaged over its channels
    plane = torch.randn(1, 1, 8, 8)
    vol = plane[:, :, None].expand(1, 1, 8, 8, 8)  # the kernel is (out, in, depth, h, w)
    w3, w2 = model.patch_embed.proj.weight, src.patch_embed.proj.weight
    out3 = torch.einsum("ocdhw,bcdhw->bo", w3, vol)
    out2 = torch.einsum("ochw,bchw->bo", w2.mean(dim=1, keepdim=True), plane)
    torch.testing.assert_close(out3, out2, atol=1e-5, rtol=1e-4)


def test_own_run_checkpoint_initialises_the_next_stage(tmp_path):
    """Stage chaining: a simmim run's DCP checkpoint directory (the whole algorithm, the encoder
    under `model.`) initialises a fresh encoder through `[init] prefix = "model."`, strictly."""
    from pathlib import Path

    from mia_train_b200 import components  # noqa: F401
    from mia_train_b200.engine.run import prepare_model, run
    from mia_train_b200.utils.config import parse_run_config

    model_kw = {"name": "dinov3_vit3d", "img_size": 16, "patch_size": 8, "embed_dim": 32, "depth": 2, "num_heads": 2}
    cfg = tmp_path / "ssl.toml"
    cfg.write_text(
        'experiment_name = "ssl"\n[model]\n' + "".join(f"{k} = {v!r}\n".replace("'", '"') for k, v in model_kw.items())
        + '[algorithm]\nname = "simmim"\nmask_ratio = 0.5\n'
        + '[data]\nname = "synthetic_volumes"\nshape = [16, 16, 16]\nsamples_per_epoch = 4\n'
        + '[trainer]\nmax_steps = 2\nbatch_size = 2\nlr = 1e-2\nwarmup_steps = 1\nprecision = "fp32"\n'
        + "checkpoint_every = 2\nlog_every = 1\n"
    )
    run_dir = Path(run(cfg, output_root=tmp_path / "runs"))
    step_dir = run_dir / "checkpoints" / "step_2"
    assert (step_dir / ".metadata").is_file()
    saved = read_state_dict(step_dir)
    config = parse_run_config({
        "experiment_name": "stage2",
        "model": model_kw,
        "init": {"path": str(step_dir), "prefix": "model.", "strict": True},
        "algorithm": {"name": "affinity_seg"},
        "data": {"name": "synthetic_volumes"},
        "trainer": {"max_steps": 1, "batch_size": 1},
    })
    model = prepare_model(config)
    key = "model.blocks.1.mlp.fc2.weight"
    assert key in saved
    torch.testing.assert_close(model.blocks[1].mlp.fc2.weight, saved[key])
