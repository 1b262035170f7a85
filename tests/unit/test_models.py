import pytest
import torch

from mia_train_b200 import components  # noqa: F401
from mia_train_b200.models.dinov3_vit import DinoVisionTransformer
from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
from mia_train_b200.models.registry import ModelRegistry
from mia_train_b200.models.vit import ViT3D
from mia_train_b200.parallel.parallel_dims import ParallelDims


def test_vit_shapes_and_flops():
    m = ViT3D(img_size=(16, 16, 32), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=2)
    x = torch.randn(2, 1, 16, 16, 32)
    tokens, grid = m.patch_features(x)
    assert tokens.shape == (2, 16, 32) and grid == (2, 2, 4)
    assert m(x).shape == (2, 32)
    assert m.flops((1, 16, 16, 32)) > 0
    with pytest.raises(ValueError):
        m.prepare_input(torch.randn(2, 2, 1, 16, 16, 32), "lcxyz")  # two scale levels


def test_vit_embed_subset_matches_full():
    torch.manual_seed(0)
    m = ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)
    x = torch.randn(2, 1, 16, 16, 16)
    full, coords = m.embed(x)
    idx = torch.tensor([[0, 3, 5], [7, 1, 2]])
    sub, sub_coords = m.embed(x, idx)
    torch.testing.assert_close(sub, torch.gather(full, 1, idx[..., None].expand(-1, -1, 32)))


def test_dinov3_3d_features_and_masks():
    m = DinoVisionTransformer3D(img_size=16, patch_size=8, embed_dim=32, depth=2, num_heads=2, n_storage_tokens=2)
    x = torch.randn(2, 1, 16, 16, 16)
    out = m.forward_features(x)
    assert out["x_norm_clstoken"].shape == (2, 32)
    assert out["x_norm_patchtokens"].shape == (2, 8, 32)
    masks = torch.zeros(2, 8, dtype=torch.bool)
    masks[:, :4] = True
    masked = m.forward_features(x, masks)
    assert not torch.allclose(masked["x_norm_patchtokens"], out["x_norm_patchtokens"])
    layers = m.get_intermediate_layers(x, n=2)
    assert len(layers) == 2


def test_windowed_equals_global_when_one_window():
    torch.manual_seed(0)
    kw = dict(img_size=16, patch_size=4, embed_dim=32, depth=2, num_heads=2, n_storage_tokens=1)
    glob = DinoVisionTransformer3D(**kw)
    win = DinoVisionTransformer3D(**kw, window_size=4)
    win.load_state_dict(glob.state_dict())
    glob.eval()
    win.eval()
    x = torch.randn(1, 1, 16, 16, 16)
    torch.testing.assert_close(win.forward_features(x)["x_norm_patchtokens"],
                               glob.forward_features(x)["x_norm_patchtokens"], atol=1e-5, rtol=1e-4)


def test_windowed_is_local():
    torch.manual_seed(0)
    m = DinoVisionTransformer3D(img_size=16, patch_size=4, embed_dim=32, depth=1, num_heads=2, window_size=2)
    m.eval()
    x = torch.randn(1, 1, 16, 16, 16)
    base = m.forward_features(x)["x_norm_patchtokens"]
    y = x.clone()
    y[..., 12:, 12:, 12:] += 1.0  # touches only the last 2^3 window of patches
    moved = (m.forward_features(y)["x_norm_patchtokens"] - base).abs().sum(-1)[0].reshape(4, 4, 4)
    # without a class token path, only the changed window's patches move
    assert moved[:2, :2, :2].max() < moved[2:, 2:, 2:].max()


def test_dinov3_2d():
    m = DinoVisionTransformer(img_size=32, patch_size=16, in_chans=1, embed_dim=32, depth=1, num_heads=2)
    out = m.forward_features(torch.randn(2, 1, 32, 32))
    assert out["x_norm_patchtokens"].shape == (2, 4, 32)


def test_block_drop_path_passes_rope_tables_through():
    """A block with drop_path > 0 in training runs the sample-subset path; with one sample the
    subset is that sample at scale 1, so the output must equal the plain (eval) path, and the shared
    per-token RoPE angles must reach the attention unchanged."""
    from mia_train_b200.layers.dinov3.block import SelfAttentionBlock
    from mia_train_b200.layers.dinov3.rope import RopePositionEmbedding3D, RopeTables

    torch.manual_seed(0)
    block = SelfAttentionBlock(32, 2, drop_path=0.5, init_values=0.5)
    rope = RopePositionEmbedding3D(32, num_heads=2)(D=2, H=2, W=2)
    assert isinstance(rope, RopeTables) and rope.angles.shape[0] == 8
    x = torch.randn(1, 9, 32)  # one prefix token + 8 patch tokens
    block.train()
    dropped = block(x, rope)
    block.eval()
    plain = block(x, rope)
    torch.testing.assert_close(dropped, plain)
    no_rope = block(x, None)
    assert not torch.allclose(plain, no_rope)

    # four samples, half of them per branch: the update lands on the drawn rows, scaled by 4 / 2
    x4 = torch.randn(4, 9, 32)
    block.train()
    torch.manual_seed(5)
    out = block(x4, rope)
    torch.manual_seed(5)
    i1, i2 = torch.randperm(4)[:2], torch.randperm(4)[:2]
    with torch.no_grad():
        mid = x4.clone()
        mid[i1] += 2 * block.ls1(block.attn(block.norm1(x4[i1]), rope=rope))
        ref = mid.clone()
        ref[i2] += 2 * block.ls2(block.mlp(block.norm2(mid[i2])))
    torch.testing.assert_close(out, ref)


def test_registry_builds_every_model():
    for name, kw in {
        "vit3d": dict(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2),
        "dinov3_vit3d": dict(img_size=16, patch_size=8, embed_dim=32, depth=1, num_heads=2),
        "dinov3_vit": dict(img_size=16, patch_size=8, embed_dim=32, depth=1, num_heads=2),
        "muvit3d": dict(levels=(1, 2), img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2),
    }.items():
        m = ModelRegistry.build(name, **kw)
        assert m.num_parameters() > 0


def test_parallel_dims_validation():
    assert ParallelDims(dp_shard=2, tp=2).world_size == 4
    assert ParallelDims(dp_replicate=2, dp_shard=2).hsdp_enabled
    with pytest.raises(ValueError):
        ParallelDims(tp=0)
    with pytest.raises(ValueError):
        ParallelDims(fsdp_unit="layer")
