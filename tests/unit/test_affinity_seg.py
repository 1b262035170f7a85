import pytest
import torch

from mia_train_b200.algorithms.affinity_seg import AffinitySegmentation
from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
from mia_train_b200.models.vit import ViT3D


def encoder():
    return ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)


@pytest.mark.parametrize("decoder", ["interpolate", "subpixel"])
@pytest.mark.parametrize("offsets", [None, "nisb12", [[1, 0, 0], [0, 0, 2]]])
def test_step_and_backward(decoder, offsets):
    alg = AffinitySegmentation(encoder(), input_axes="lcxyz", decoder=decoder, offsets=offsets,
                               decoder_hidden_dim=8, decoder_zero_init_output=False)
    batch = {"img": torch.randn(2, 1, 1, 16, 16, 16), "label": torch.randint(0, 3, (2, 1, 16, 16, 16))}
    out = alg(batch)
    assert set(out) >= {"loss", "affinity_accuracy", "boundary_accuracy", "target_positive_rate", "masked_fraction"}
    out["loss"].backward()
    assert alg.decoder_out.out.weight.grad is not None if decoder == "subpixel" else True


def test_axis_order_enforced():
    with pytest.raises(ValueError, match="x,y,z"):
        AffinitySegmentation(encoder(), input_axes="lczyx")


def test_label_checks():
    alg = AffinitySegmentation(encoder(), input_axes="lcxyz", decoder_hidden_dim=8)
    with pytest.raises(KeyError):
        alg({"img": torch.randn(1, 1, 1, 16, 16, 16)})
    with pytest.raises(ValueError, match="single-scale"):
        alg({"img": torch.randn(1, 1, 1, 16, 16, 16), "label": torch.zeros(1, 2, 16, 16, 16, dtype=torch.long)})


def test_sample_transform_delegates_split():
    alg = AffinitySegmentation(encoder(), input_axes="lcxyz", decoder_hidden_dim=8)
    assert alg.sample_transform() is not None and alg._split_delegated
    alg2 = AffinitySegmentation(encoder(), input_axes="lcxyz", decoder_hidden_dim=8, split_disconnected=False)
    assert alg2.sample_transform() is None


def test_dinov3_encoder_subpixel():
    enc = DinoVisionTransformer3D(img_size=16, patch_size=8, embed_dim=32, depth=1, num_heads=2)
    alg = AffinitySegmentation(enc, input_axes="lcxyz", decoder="subpixel", decoder_hidden_dim=8)
    out = alg({"img": torch.randn(1, 1, 1, 16, 16, 16), "label": torch.randint(0, 3, (1, 1, 16, 16, 16))})
    out["loss"].backward()
