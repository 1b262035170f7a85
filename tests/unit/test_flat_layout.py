"""Flat parameter layout used by the captured step and the sharded optimizer (CPU-only checks)."""

import pytest
import torch
import torch.nn as nn

from mia_train_b200.engine.graph_step import FlatParameters, _overlap_blocks
from mia_train_b200.models.vit import ViT3D


def model():
    return ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=3, num_heads=2)


@pytest.mark.parametrize("world", [1, 2, 8])
def test_segments_partition_and_align(world):
    m = model()
    groups = [list(b.parameters()) for b in _overlap_blocks(m)]
    before = {n: p.detach().clone() for n, p in m.named_parameters()}
    flat = FlatParameters(m, world=world, bf16_region=True, groups=groups)
    unit = 64 * world
    assert flat.segments[0][0] == 0 and flat.segments[-1][1] == flat.total
    for (a, b), (c, _) in zip(flat.segments, flat.segments[1:]):
        assert b == c
    assert all((b - a) % unit == 0 for a, b in flat.segments)
    assert all(off % 64 == 0 for off in flat.offsets)
    # GEMM weights (Linear / conv) live at or after bf16_begin, everything else before it
    gemm = {id(mod.weight) for mod in m.modules() if isinstance(mod, (nn.Linear, nn.modules.conv._ConvNd))}
    for p, off in zip(flat.params, flat.offsets):
        assert (off >= flat.bf16_begin) == (id(p) in gemm)
    # parameters keep their values and become views of the flat buffers
    for n, p in m.named_parameters():
        torch.testing.assert_close(p.detach(), before[n])
        assert p.main_grad.shape == p.shape
    assert len(flat.groups) == 3  # one segment per transformer block
    flat.release()
    assert not any(hasattr(p, "main_grad") for p in m.parameters())


def test_without_bf16_region_everything_is_fp32():
    m = model()
    flat = FlatParameters(m, world=4)
    assert flat.bf16_begin == flat.total and len(flat.segments) == 1
