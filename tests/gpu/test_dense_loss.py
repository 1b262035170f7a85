"""Fused dense-loss kernels and the multi-tensor EMA against fp32 PyTorch references."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU collection
    pytest.skip("needs CUDA", allow_module_level=True)

from mia_train_b200.algorithms.affinity.targets import affinity_offsets, offset_preset  # noqa: E402
from mia_train_b200.ops import _native  # noqa: E402
from mia_train_b200.ops.dense_loss import (  # noqa: E402
    affinity_bce,
    affinity_bce_reference,
    semantic_ce,
    semantic_ce_reference,
)
from mia_train_b200.ops.optim import ema_update  # noqa: E402


@pytest.fixture(autouse=True)
def _loaded():
    _native.native()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("offsets", ["default", "nisb12", "negative"])
@pytest.mark.parametrize("shape", [(2, 16, 16, 16), (1, 7, 12, 9)])
def test_affinity_bce_matches_reference(dtype, offsets, shape):
    torch.manual_seed(0)
    offs = {"default": affinity_offsets(3, 4), "nisb12": offset_preset("nisb12"),
            "negative": ((-1, 0, 0), (0, -2, 1), (3, 3, 0))}[offsets]
    labels = torch.randint(-1, 4, shape, device="cuda")
    logits = torch.randn(shape[0], len(offs), *shape[1:], device="cuda").to(dtype).requires_grad_(True)
    ref_logits = logits.detach().float().requires_grad_(True)
    got = affinity_bce(logits, labels, offs, ignore_index=-1)
    ref = affinity_bce_reference(ref_logits, labels, offs, ignore_index=-1)
    for key in ref:
        torch.testing.assert_close(got[key].float(), ref[key].float(), atol=2e-5, rtol=1e-4, msg=key)
    got["loss"].backward()
    ref["loss"].backward()
    tol = 1e-6 if dtype == torch.float32 else 2e-3
    torch.testing.assert_close(logits.grad.float(), ref_logits.grad, atol=tol, rtol=1e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize("spatial", [(16, 16, 16), (33, 20)])
def test_semantic_ce_matches_reference(dtype, weighted, spatial):
    torch.manual_seed(1)
    k = 7
    labels = torch.randint(-1, k, (2, *spatial), device="cuda")
    logits = (3 * torch.randn(2, k, *spatial, device="cuda")).to(dtype).requires_grad_(True)
    ref_logits = logits.detach().float().requires_grad_(True)
    w = torch.rand(k, device="cuda") + 0.5 if weighted else None
    got = semantic_ce(logits, labels, w, -1)
    ref = semantic_ce_reference(ref_logits, labels, w, -1)
    for key in ref:
        torch.testing.assert_close(got[key].float(), ref[key].float(), atol=1e-5, rtol=1e-4, msg=key)
    got["loss"].backward()
    ref["loss"].backward()
    tol = 1e-6 if dtype == torch.float32 else 2e-3
    torch.testing.assert_close(logits.grad.float(), ref_logits.grad, atol=tol, rtol=1e-2)


def test_ema_update_matches_foreach():
    torch.manual_seed(2)
    shapes = [(1000,), (33, 17), (4096, 4), (5,)]
    teacher = [torch.randn(s, device="cuda") for s in shapes]
    student = [torch.randn(s, device="cuda") for s in shapes]
    expect = [0.994 * t + 0.006 * s for t, s in zip(teacher, student, strict=True)]
    ema_update(teacher, student, 0.994)
    for t, e in zip(teacher, expect, strict=True):
        torch.testing.assert_close(t, e, atol=1e-6, rtol=1e-6)
    assert _native.native().check_errors(0) == 0
