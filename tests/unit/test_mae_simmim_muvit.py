import pytest
import torch

from mia_train_b200.algorithms.mae import MAE
from mia_train_b200.algorithms.muvit_mae import MuViTMAE
from mia_train_b200.algorithms.simmim import SimMIM, patchify, random_mask
from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
from mia_train_b200.models.muvit import MuViT3D
from mia_train_b200.models.vit import ViT3D


def vit(**kw):
    args = dict(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=2)
    args.update(kw)
    return ViT3D(**args)


def test_mae_masking_keeps_ratio():
    alg = MAE(vit(img_size=(32, 32, 32)), input_axes="lcxyz", mask_ratio=0.75, decoder_embed_dim=16,
              decoder_depth=1, decoder_num_heads=2)
    out = alg({"img": torch.randn(2, 1, 1, 32, 32, 32)})
    assert float(out["masked_fraction"]) == pytest.approx(0.75)
    out["loss"].backward()


@pytest.mark.parametrize("pos_embed", ["rope", "sincos", "learned"])
def test_mae_position_variants(pos_embed):
    alg = MAE(vit(pos_embed=pos_embed), input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    out = alg({"img": torch.randn(2, 1, 1, 16, 16, 16)})
    assert torch.isfinite(out["loss"])


def test_mae_rejects_multiscale():
    alg = MAE(vit(), input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    with pytest.raises(ValueError):
        alg({"img": torch.randn(2, 2, 1, 16, 16, 16)})


def test_patchify_roundtrip_order():
    v = torch.arange(2 * 1 * 4 * 4 * 4, dtype=torch.float32).reshape(2, 1, 4, 4, 4)
    rows = patchify(v, (2, 2, 2))
    assert rows.shape == (2, 8, 8)
    assert rows[0, 0].tolist() == [0, 1, 4, 5, 16, 17, 20, 21]


def test_random_mask_granularity():
    m = random_mask((4, 4, 4), 3, 0.5, granularity=2)
    assert m.shape == (3, 64)
    grid = m.reshape(3, 4, 4, 4)
    # 2x2x2 units are all-or-nothing
    units = grid.reshape(3, 2, 2, 2, 2, 2, 2).permute(0, 1, 3, 5, 2, 4, 6).reshape(3, 8, 8)
    assert ((units.all(-1)) | (~units.any(-1))).all()


def test_simmim_step():
    enc = DinoVisionTransformer3D(img_size=16, patch_size=4, embed_dim=32, depth=1, num_heads=2)
    alg = SimMIM(enc, input_axes="lcxyz", mask_ratio=0.5, mask_granularity=2)
    out = alg({"img": torch.randn(2, 1, 1, 16, 16, 16)})
    assert "loss" in out
    out["loss"].backward()
    assert enc.mask_token.grad is not None


def test_muvit_mae_step():
    enc = MuViT3D(levels=(1, 2), img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)
    alg = MuViTMAE(enc, input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    bbox = enc.default_bbox(2, torch.device("cpu"))
    out = alg({"img": torch.randn(2, 2, 1, 16, 16, 16), "bbox": bbox})
    out["loss"].backward()
    with pytest.raises(KeyError, match="bbox"):
        alg({"img": torch.randn(2, 2, 1, 16, 16, 16)})


def test_muvit_level_checks():
    with pytest.raises(ValueError, match="finest first"):
        MuViT3D(levels=(4, 1), img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)
    with pytest.raises(ValueError, match="distinct"):
        MuViT3D(levels=(1, 1), img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)
