import pytest
import torch

from mia_train_b200.algorithms.semantic_seg import SemanticSegmentation
from mia_train_b200.models.dinov3_vit import DinoVisionTransformer
from mia_train_b200.models.vit import ViT3D
from mia_train_b200.ops.dense_loss import semantic_ce_reference


def test_3d_step_weights_and_checkpointed_decoder():
    enc = ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)
    alg = SemanticSegmentation(enc, input_axes="lcxyz", num_classes=4, decoder_hidden_dim=8,
                               class_weights=[1.0, 2.0, 1.0, 0.5], checkpoint_decoder=True)
    out = alg({"img": torch.randn(2, 1, 1, 16, 16, 16), "label": torch.randint(-1, 4, (2, 1, 16, 16, 16))})
    assert set(out) == {"loss", "pixel_accuracy", "mean_iou", "classes_present"}
    out["loss"].backward()
    assert "class_weights" in alg.state_dict()


def test_2d_model():
    enc = DinoVisionTransformer(img_size=16, patch_size=8, in_chans=1, embed_dim=32, depth=1, num_heads=2)
    alg = SemanticSegmentation(enc, input_axes="lcxy", num_classes=3, decoder_hidden_dim=8)
    assert alg.spatial_rank == 2
    out = alg({"img": torch.randn(2, 1, 1, 16, 16), "label": torch.randint(0, 3, (2, 1, 16, 16))})
    out["loss"].backward()


def test_validation():
    enc = ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=1, num_heads=2)
    with pytest.raises(ValueError):
        SemanticSegmentation(enc, input_axes="lcxyz", num_classes=1)
    with pytest.raises(ValueError, match="class_weights"):
        SemanticSegmentation(enc, input_axes="lcxyz", num_classes=3, class_weights=[1.0])


def test_reference_metrics_by_hand():
    logits = torch.tensor([[[[5.0, 0.0]], [[0.0, 5.0]]]])  # (1, 2 classes, 1, 2)
    labels = torch.tensor([[[0, 0]]])
    out = semantic_ce_reference(logits, labels)
    assert out["pixel_accuracy"] == pytest.approx(0.5)
    assert out["mean_iou"] == pytest.approx(0.5)  # class 0: 1 / 2
    assert out["classes_present"] == 1
