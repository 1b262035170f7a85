import pytest
import torch

from mia_train_b200.algorithms.affinity.targets import (
    SplitDisconnectedLabels,
    affinities_from_labels,
    affinity_offsets,
    offset_preset,
    relabel_connected,
    relabel_connected_host,
)
from mia_train_b200.ops.dense_loss import affinity_bce, affinity_bce_reference


def same_partition(a: torch.Tensor, b: torch.Tensor) -> bool:
    pairs = set(zip(a.flatten().tolist(), b.flatten().tolist()))
    return len(pairs) == len(set(a.flatten().tolist())) == len(set(b.flatten().tolist()))


def test_default_offsets_order():
    assert affinity_offsets(3, 10) == ((1, 0, 0), (0, 1, 0), (0, 0, 1), (10, 0, 0), (0, 10, 0), (0, 0, 10))
    assert affinity_offsets(2, 4) == ((1, 0), (0, 1), (4, 0), (0, 4))


def test_nisb12_preset():
    offs = offset_preset("nisb12")
    assert len(offs) == 12 and max(max(o) for o in offs) == 9
    assert offs[:3] == ((1, 0, 0), (0, 1, 0), (0, 0, 1))
    with pytest.raises(KeyError):
        offset_preset("nope")


def test_targets_semantics():
    labels = torch.tensor([[[1, 1, 0, 2, 2, -1]]])  # (B=1, 1, 6): rank 2 with a singleton axis
    target, mask = affinities_from_labels(labels, ((0, 1),), ignore_index=-1)
    assert target[0, 0, 0].tolist() == [True, False, False, True, False, False]
    # last column has no neighbour; the pair (2, -1) touches ignore
    assert mask[0, 0, 0].tolist() == [True, True, True, True, False, False]


def test_background_never_affine():
    labels = torch.zeros(1, 4, 4, dtype=torch.long)
    target, mask = affinities_from_labels(labels, ((1, 0), (0, 1)))
    assert not target.any() and mask.sum() == 2 * 3 * 4


def test_relabel_splits_disconnected_pieces():
    labels = torch.zeros(8, 8, 8, dtype=torch.long)
    labels[1] = 3
    labels[5] = 3
    labels[3, 3, 3] = -1
    out = relabel_connected(labels)
    assert out[1].unique().numel() == 1 and out[5].unique().numel() == 1
    assert out[1, 0, 0] != out[5, 0, 0]
    assert out[3, 3, 3] == -1 and out[0, 0, 0] == 0


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_host_and_device_labelling_agree(seed):
    g = torch.Generator().manual_seed(seed)
    labels = torch.randint(-1, 3, (12, 10, 9), generator=g)
    assert same_partition(relabel_connected(labels), relabel_connected_host(labels))


def test_split_transform_runs_per_level():
    labels = torch.zeros(2, 6, 6, 6, dtype=torch.int32)
    labels[:, 0] = 1
    labels[:, 4] = 1
    out = SplitDisconnectedLabels("label")({"label": labels, "img": torch.zeros(1)})
    assert out["label"].dtype == torch.int32
    assert out["label"][0, 0, 0, 0] != out["label"][0, 4, 0, 0]
    with pytest.raises(KeyError):
        SplitDisconnectedLabels("label")({"img": torch.zeros(1)})


def test_loss_reference_and_dispatch_agree_on_cpu():
    torch.manual_seed(0)
    labels = torch.randint(0, 3, (1, 6, 6, 6))
    logits = torch.randn(1, 6, 6, 6, 6)
    a = affinity_bce(logits, labels, affinity_offsets(3, 2))
    b = affinity_bce_reference(logits, labels, affinity_offsets(3, 2))
    for k in b:
        torch.testing.assert_close(a[k], b[k])
