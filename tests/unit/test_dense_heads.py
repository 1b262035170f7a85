import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from mia_train_b200.layers.common.dense_heads import SubPixelHead, VoxelHead, linear_resample_matrix


@pytest.mark.parametrize("extent,target", [(8, 128), (5, 17), (16, 16), (7, 3), (1, 4)])
def test_resample_matrix_matches_interpolate(extent, target):
    m = linear_resample_matrix(extent, target).double()
    basis = torch.eye(extent, dtype=torch.float64).reshape(extent, 1, extent)
    ref = F.interpolate(basis, size=target, mode="linear", align_corners=False).squeeze(1).T
    torch.testing.assert_close(m, ref, atol=1e-6, rtol=0)


@pytest.mark.parametrize("size", [(9, 8, 10), (16, 16, 16)])
def test_voxel_head_upsample_is_trilinear(size):
    head = VoxelHead(nn.Identity())
    x = torch.randn(2, 3, 3, 4, 5)
    ref = F.interpolate(x.double(), size=size, mode="trilinear", align_corners=False)
    torch.testing.assert_close(head.upsample(x, size).double(), ref, atol=1e-5, rtol=0)
    assert head(x, size).shape == (2, 3, *size)


def test_voxel_head_2d():
    head = VoxelHead(nn.Conv2d(3, 2, 1), mode="bilinear")
    x = torch.randn(1, 3, 4, 6)
    ref = F.interpolate(x, size=(8, 12), mode="bilinear", align_corners=False)
    torch.testing.assert_close(head.upsample(x, (8, 12)), ref, atol=1e-5, rtol=0)


@pytest.mark.parametrize("patch", [(4, 4, 4), (2, 3, 4), (4, 2)])
def test_subpixel_gemm_equals_transposed_conv(patch):
    head = SubPixelHead(8, patch, 3, hidden=6, readout=5, zero_init_output=False)
    grid = (3, 2, 5)[: len(patch)]
    x = torch.randn(2, 6, *grid)
    torch.testing.assert_close(head.expand_tokens(x), head.expand(x), atol=1e-5, rtol=1e-5)


def test_subpixel_rejects_partial_patches_and_zero_inits():
    head = SubPixelHead(8, (4, 4, 4), 3, hidden=6, readout=5)
    x = torch.randn(1, 8, 2, 2, 2)
    with pytest.raises(ValueError, match="divisible"):
        head(x, (8, 8, 9))
    out = head(x, (8, 8, 8))
    assert torch.count_nonzero(out) == 0  # zero-initialised output layer and bias
    head.set_output_bias(-2.0)
    assert torch.allclose(head(x, (8, 8, 8)), torch.full_like(out, -2.0))
    with pytest.raises(ValueError, match="refine_depth"):
        SubPixelHead(8, (4, 4, 4), 3, refine_depth=0)
