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
