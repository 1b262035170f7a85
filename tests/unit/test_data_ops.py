"""CPU path of the device-side input normalisation."""

from __future__ import annotations

import pytest
import torch

from mia_train_b200.ops.data import zscore_u8


def test_zscore_u8_cpu_matches_formula():
    x = torch.randint(0, 256, (3, 1, 8, 8, 8), dtype=torch.uint8)
    y = zscore_u8(x, torch.float32)
    v = x.double().flatten(1)
    ref = (v - v.mean(1, keepdim=True)) / v.std(1, keepdim=True)
    torch.testing.assert_close(y.flatten(1).double(), ref, atol=1e-5, rtol=1e-5)


def test_zscore_u8_rejects_float_input():
    with pytest.raises(TypeError):
        zscore_u8(torch.zeros(2, 16), torch.float32)
