import pytest
import torch
import torch.nn as nn

from mia_train_b200.evals.semantic_seg import (
    ConfusionMatrix,
    SemanticSegmentationEval,
    blend_weight,
    orthoplane_logits,
    tile_starts,
    tiled_logits,
)


def test_tile_starts_cover_and_pull_back():
    assert tile_starts(10, 16, 2) == [0]
    assert tile_starts(10, 4, 0) == [0, 3, 6]  # the fewest tiles, spread evenly
    for extent, tile, overlap in ((100, 32, 8), (257, 64, 16), (64, 64, 0), (65, 64, 32)):
        s = tile_starts(extent, tile, overlap)
        assert s[0] == 0 and s[-1] == max(0, extent - tile)
        assert all(0 < b - a <= tile - overlap for a, b in zip(s, s[1:]))  # at least `overlap` overlap


def test_blend_weight_profile():
    w = blend_weight((5,), torch.device("cpu"))
    assert w.tolist() == [1.0, 2.0, 3.0, 2.0, 1.0]


def test_tiled_identity_predictor_is_exact():
    k = 3

    def predict(x):  # one-hot of a deterministic function of the voxel value
        return torch.cat([x * (i + 1) for i in range(k)], dim=1)

    img = torch.rand(2, 10, 12)
    out = tiled_logits(predict, img, (4, 5), 2, k, torch.device("cpu"))
    expect = torch.stack([img * (i + 1) for i in range(k)], dim=1)
    torch.testing.assert_close(out, expect, atol=1e-5, rtol=1e-5)


def test_orthoplane_averages_three_axes():
    vol = torch.rand(4, 5, 6)
    out = orthoplane_logits(lambda x: torch.cat([x, -x], dim=1), vol, (8, 8), 0, 2, torch.device("cpu"))
    torch.testing.assert_close(out[0], vol, atol=1e-5, rtol=1e-5)


def test_confusion_metrics():
    cm = ConfusionMatrix(3)
    cm.update(torch.tensor([0, 1, 1, 2, 2]), torch.tensor([0, 1, 2, 2, -1]), ignore_index=-1)
    m = cm.metrics()
    assert m["pixel_accuracy"] == pytest.approx(3 / 4)
    assert m["classes_present"] == 3
    assert m["iou/class_1"] == pytest.approx(1 / 2)
    assert m["mean_iou"] == pytest.approx((1 + 0.5 + 0.5) / 3)


class Fake(nn.Module):
    spatial_rank = 3

    def logits(self, x):
        return torch.cat([1 - x, x], dim=1)


def test_eval_task_end_to_end():
    task = SemanticSegmentationEval(num_classes=2, tile=(8, 8, 8), overlap=2, device="cpu")
    img = (torch.rand(1, 1, 1, 12, 12, 12) > 0.5).float()
    batch = {"img": img, "label": img[:, 0, 0].long().unsqueeze(1)}
    m = task.evaluate(Fake(), [batch])
    assert m["pixel_accuracy"] == pytest.approx(1.0)
    with pytest.raises(ValueError, match="orthoplane"):
        SemanticSegmentationEval(num_classes=2, tile=(8, 8, 8), mode="orthoplane").evaluate(Fake(), [batch])
