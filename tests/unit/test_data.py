import pytest
import torch

from mia_train_b200.data.augment import VolumeAugmentation
from mia_train_b200.data.huggingface import HuggingFaceSemanticSegmentation, group_of, random_crop
from mia_train_b200.data.synthetic import SyntheticVolumes


@pytest.mark.parametrize("generator", ["noise", "blobs", "voronoi"])
def test_synthetic_reproducible(generator):
    ds = SyntheticVolumes(generator=generator, shape=(16, 16, 16), samples_per_epoch=4, seed=3, n_seeds=10, blob_rate=5.0)
    a = ds.dataset[1]
    b = SyntheticVolumes(generator=generator, shape=(16, 16, 16), samples_per_epoch=4, seed=3, n_seeds=10,
                         blob_rate=5.0).dataset[1]
    assert a["img"].shape == (1, 1, 16, 16, 16)
    torch.testing.assert_close(a["img"], b["img"])
    assert not torch.equal(a["img"], ds.dataset[2]["img"])
    if generator == "voronoi":
        assert a["label"].shape == (1, 16, 16, 16) and (a["label"] == 0).any()
    assert ds.sample_axes == "lcxyz"


def test_synthetic_rejects_unknown():
    with pytest.raises(ValueError):
        SyntheticVolumes(generator="fractal")
    with pytest.raises(ValueError):
        SyntheticVolumes.resolve_settings(bogus=1)


def test_synthetic_pyramid_levels_agree_and_boxes_are_concentric():
    ds = SyntheticVolumes(generator="noise", shape=(16, 16, 16), levels=(1, 2, 8), samples_per_epoch=2, seed=3)
    sample = ds.dataset[1]
    img, bbox = sample["img"], sample["bbox"]
    assert img.shape == (3, 1, 16, 16, 16) and bbox.shape == (3, 2, 3)
    torch.testing.assert_close(ds.dataset[1]["img"], img)  # deterministic in (seed, index)
    centres = bbox.mean(dim=1)
    torch.testing.assert_close(centres, centres[:1].expand(3, 3))
    spans = bbox[:, 1] - bbox[:, 0]
    torch.testing.assert_close(spans, torch.tensor([[1.0], [2.0], [8.0]]) * 15.0 * torch.ones(3, 3))
    # level 0 is level 1's central half, upsampled, plus fresh detail: the two correlate
    centre = img[1, 0, 4:12, 4:12, 4:12]
    up = torch.nn.functional.interpolate(centre[None, None], size=(16, 16, 16), mode="trilinear")[0, 0]
    corr = torch.corrcoef(torch.stack((img[0, 0].flatten(), up.flatten())))[0, 1]
    assert corr > 0.2


def test_synthetic_levels_validation():
    with pytest.raises(ValueError, match="levels"):
        SyntheticVolumes(levels=(1, 3, 4))
    with pytest.raises(ValueError, match="levels"):
        SyntheticVolumes(levels=(2, 1))
    with pytest.raises(ValueError, match="noise or blobs"):
        SyntheticVolumes(generator="voronoi", levels=(1, 2))
    with pytest.raises(ValueError, match="divide"):
        SyntheticVolumes(shape=(30, 32, 32), levels=(1, 4))


def test_synthetic_semantic_classes():
    ds = SyntheticVolumes(generator="voronoi", shape=(16, 16, 16), n_seeds=20, classes=4)
    sample = ds.dataset[0]
    labels, img = sample["label"][0], sample["img"][0, 0]
    assert set(labels.unique().tolist()) <= {0, 1, 2, 3} and labels.max() > 0
    # the mean intensity rises with the class (away from boundaries, where the blur mixes cells)
    means = [img[labels == c].mean() for c in (1, 2, 3) if (labels == c).sum() > 20]
    assert all(a < b for a, b in zip(means, means[1:], strict=False))
    with pytest.raises(ValueError, match="classes"):
        SyntheticVolumes(generator="noise", classes=3)
    with pytest.raises(ValueError, match="classes"):
        SyntheticVolumes(generator="voronoi", classes=1)


def test_dataloader_shards_by_dp_rank():
    ds = SyntheticVolumes(shape=(8, 8, 8), samples_per_epoch=8)
    loaders = [ds.build_dataloader(batch_size=2, rank=r, world_size=2, num_workers=0, shuffle=False)
               for r in range(2)]
    seen = [torch.cat([b["img"] for b in dl]) for dl in loaders]
    assert seen[0].shape[0] == seen[1].shape[0] == 4
    assert not torch.equal(seen[0], seen[1])


def test_transform_attach_after_build_refused():
    ds = SyntheticVolumes(shape=(8, 8, 8), samples_per_epoch=2)
    ds.attach_transform(lambda s: s)
    _ = ds.dataset
    with pytest.raises(RuntimeError):
        ds.attach_transform(lambda s: s)


def test_augment_rotation_keeps_label_alignment():
    torch.manual_seed(0)
    aug = VolumeAugmentation(rotate="full", sample_axes="lcxyz")
    img = torch.arange(8 * 8 * 8, dtype=torch.float32).reshape(1, 1, 8, 8, 8)
    label = img[:, 0].long()
    for _ in range(5):
        out = aug({"img": img.clone(), "label": label.clone()})
        assert torch.equal(out["img"][:, 0].long(), out["label"])


def test_augment_validation():
    with pytest.raises(ValueError):
        VolumeAugmentation(rotate="sideways")
    with pytest.raises(ValueError):
        VolumeAugmentation(rotate="full")  # needs the axis order
    with pytest.raises(ValueError):
        VolumeAugmentation(drop_slice_prob=2.0)


def test_hf_helpers_and_presets():
    import numpy as np

    assert group_of("jrc_hela-2/recon-1/crop28", 1) == "jrc_hela-2"
    assert group_of("jrc_hela-2/recon-1/crop28", 2) == "jrc_hela-2/recon-1"
    img, lab = random_crop(np.ones((3, 5)), np.ones((3, 5)), (4, 4), np.random.default_rng(0))
    assert img.shape == (4, 4) and img[3].sum() == 0
    ds = HuggingFaceSemanticSegmentation(patch_size=(16, 16, 16), preset="cellmap_3d")
    assert ds.sample_axes == "lcxyz"
    settings = HuggingFaceSemanticSegmentation.resolve_settings(patch_size=(16, 16, 16), preset="cellmap_3d")
    assert settings["repo"] == "eminorhan/cellmap-3d"
    with pytest.raises(ValueError):
        HuggingFaceSemanticSegmentation(patch_size=(16, 16), preset="cellmap_3d")
    with pytest.raises(ValueError, match="hold_out"):
        HuggingFaceSemanticSegmentation(patch_size=(16, 16, 16), preset="cellmap_3d", split="val")


def test_hf_row_selection_by_group():
    class Table:
        def __init__(self, rows):
            self.rows = rows
            self.column_names = list(rows[0])

        def __getitem__(self, key):
            return [r[key] for r in self.rows] if isinstance(key, str) else self.rows[key]

        def select(self, idx):
            return Table([self.rows[i] for i in idx])

        def __len__(self):
            return len(self.rows)

    rows = Table([{"crop_name": f"s{i % 3}/r/c{i}", "axis": "xyz"[i % 3]} for i in range(9)])
    val = HuggingFaceSemanticSegmentation(patch_size=(8, 8), preset="cellmap_2d", hold_out_groups=["s1"], split="val")
    train = HuggingFaceSemanticSegmentation(patch_size=(8, 8), preset="cellmap_2d", hold_out_groups=["s1"],
                                            row_filters={"axis": ["x", "y"]})
    assert {r["crop_name"][:2] for r in val.select_rows(rows).rows} == {"s1"}
    kept = train.select_rows(rows).rows
    assert all(r["crop_name"][:2] == "s0" for r in kept)


def test_miao_missing_is_clear():
    from mia_train_b200.data.miao_dataset import MiaoVolumeDataset

    try:
        import miao  # noqa: F401
    except ImportError:
        with pytest.raises(ImportError, match="miao"):
            MiaoVolumeDataset(output_axes="lcxyz")
