"""Fused dense-prediction losses (affinity BCE, semantic CE) and host connected components.

`affinity_bce(logits, labels, offsets, ignore_index)` returns the masked mean BCE-with-logits of
affinity logits against targets derived from instance labels, plus the reference's metrics
(accuracy, boundary accuracy, positive rate, masked fraction), without materialising the target or
mask tensors (reference `src/algorithms/affinity_seg.py:298-323`, targets
`src/algorithms/affinity/targets.py:213-260`). On CUDA it is two kernels (forward statistics,
backward gradient); elsewhere the PyTorch reference below runs.

`semantic_ce(logits, labels, weights, ignore_index)` returns the weighted-mean cross-entropy plus
pixel accuracy, mean IoU over the classes present, and their count (reference
`src/algorithms/semantic_seg.py:194-217`), with argmax and the per-class intersection / union
histogram computed in the same pass as the loss.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
import torch.nn.functional as F

from ._native import native, use_native


def _flat_offsets(offsets: Sequence[Sequence[int]]) -> list[int]:
    flat: list[int] = []
    for o in offsets:
        if len(o) != 3:
            raise ValueError(f"native affinity offsets are 3-D, got {tuple(o)}")
        flat += [int(v) for v in o]
    return flat


def offset_slices(offset: Sequence[int], spatial: Sequence[int]) -> tuple[tuple[slice, ...], tuple[slice, ...]]:
    """Source and shifted-target regions related by `offset`; outside them there is no neighbour."""
    src, dst = [], []
    for d, n in zip(offset, spatial, strict=True):
        keep = max(n - abs(d), 0)
        if d >= 0:
            src.append(slice(0, keep))
            dst.append(slice(d, d + keep))
        else:
            src.append(slice(-d, -d + keep))
            dst.append(slice(0, keep))
    return tuple(src), tuple(dst)


def affinity_targets_reference(
    labels: torch.Tensor, offsets: Sequence[Sequence[int]], ignore_index: int = -1
) -> tuple[torch.Tensor, torch.Tensor]:
    """(B, *S) ids -> bool (target, mask), each (B, len(offsets), *S)."""
    if labels.ndim < 2:
        raise ValueError(f"labels must be (B, *spatial), got {tuple(labels.shape)}")
    rank = labels.ndim - 1
    shape = (labels.shape[0], len(offsets), *labels.shape[1:])
    target = torch.zeros(shape, dtype=torch.bool, device=labels.device)
    mask = torch.zeros_like(target)
    known = labels != ignore_index
    for c, off in enumerate(offsets):
        if len(off) != rank:
            raise ValueError(f"offset {tuple(off)} has {len(off)} components but labels have {rank} spatial axes")
        s, d = offset_slices(off, labels.shape[1:])
        a = labels[(slice(None), *s)]
        b = labels[(slice(None), *d)]
        target[(slice(None), c, *s)] = (a == b) & (a > 0)
        mask[(slice(None), c, *s)] = known[(slice(None), *s)] & known[(slice(None), *d)]
    return target, mask


def affinity_bce_reference(
    logits: torch.Tensor, labels: torch.Tensor, offsets: Sequence[Sequence[int]], ignore_index: int = -1
) -> dict[str, torch.Tensor]:
    target, mask = affinity_targets_reference(labels, offsets, ignore_index)
    t = target.float()
    per = F.binary_cross_entropy_with_logits(logits.float(), t, reduction="none")
    den = mask.sum().clamp_min(1.0)
    loss = (per * mask).sum() / den
    with torch.no_grad():
        correct = ((logits > 0) == target) & mask
        cut = mask & ~target
        out = {
            "affinity_accuracy": correct.sum() / den,
            "boundary_accuracy": (correct & cut).sum() / cut.sum().clamp_min(1.0),
            "target_positive_rate": (t * mask).sum() / den,
            "masked_fraction": mask.float().mean(),
        }
    return {"loss": loss, **out}


class _AffinityLoss(torch.autograd.Function):
    """loss = sums[0] / max(sums[1], 1); the backward feeds the scalar grad to the fused kernel."""

    @staticmethod
    def forward(ctx, logits, labels, flat, ignore_index):
        sums = native().affinity_bce_fwd(logits, labels, flat, ignore_index)
        ctx.save_for_backward(logits, labels, sums)
        ctx.flat, ctx.ignore = flat, ignore_index
        ctx.mark_non_differentiable(sums)
        loss = (sums[0] / sums[1].clamp_min(1.0)).float()
        return loss, sums

    @staticmethod
    def backward(ctx, g_loss, _g_sums):
        logits, labels, sums = ctx.saved_tensors
        g = g_loss.float().reshape(1).contiguous()
        grad = native().affinity_bce_bwd(logits, labels, ctx.flat, ctx.ignore, sums, g)
        return grad, None, None, None


def affinity_bce(
    logits: torch.Tensor, labels: torch.Tensor, offsets: Sequence[Sequence[int]], ignore_index: int = -1
) -> dict[str, torch.Tensor]:
    native_ok = (
        logits.dim() == 5
        and logits.dtype in (torch.bfloat16, torch.float32)
        and labels.dtype in (torch.int64, torch.int32)
        and all(len(o) == 3 for o in offsets)
        and use_native(logits, labels)
    )
    if not native_ok:
        return affinity_bce_reference(logits, labels, offsets, ignore_index)
    loss, sums = _AffinityLoss.apply(logits.contiguous(), labels.contiguous(), _flat_offsets(offsets), int(ignore_index))
    s = sums.float()
    den = s[1].clamp_min(1.0)
    return {
        "loss": loss,
        "affinity_accuracy": s[2] / den,
        "boundary_accuracy": s[5] / s[4].clamp_min(1.0),
        "target_positive_rate": s[3] / den,
        "masked_fraction": s[1] / float(logits.numel()),
    }


# ---------------------------------------------------------------------------------------------
def semantic_ce_reference(
    logits: torch.Tensor, labels: torch.Tensor, weights: torch.Tensor | None = None, ignore_index: int = -1
) -> dict[str, torch.Tensor]:
    loss = F.cross_entropy(logits.float(), labels, weight=weights, ignore_index=ignore_index)
    with torch.no_grad():
        pred = logits.argmax(dim=1)
        valid = labels != ignore_index
        den = valid.sum().clamp_min(1)
        acc = ((pred == labels) & valid).sum() / den
        ious = []
        for k in torch.unique(labels[valid]):
            p, t = (pred == k) & valid, (labels == k) & valid
            ious.append((p & t).sum() / (p | t).sum().clamp_min(1))
        miou = torch.stack(ious).mean() if ious else torch.tensor(float("nan"), device=logits.device)
    return {"loss": loss, "pixel_accuracy": acc, "mean_iou": miou,
            "classes_present": torch.tensor(float(len(ious)), device=logits.device)}


class _SemanticCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, weights, ignore_index):
        stats, hist = native().semantic_ce_fwd(logits, labels, weights, ignore_index)
        ctx.save_for_backward(logits, labels, stats, *( [weights] if weights is not None else []))
        ctx.has_w, ctx.ignore = weights is not None, ignore_index
        ctx.mark_non_differentiable(stats, hist)
        return (stats[0] / stats[1]).float(), stats, hist

    @staticmethod
    def backward(ctx, g_loss, _gs, _gh):
        saved = ctx.saved_tensors
        logits, labels, stats = saved[:3]
        weights = saved[3] if ctx.has_w else None
        grad = native().semantic_ce_bwd(logits, labels, weights, ctx.ignore, stats, g_loss.float().reshape(1).contiguous())
        return grad, None, None, None


def semantic_ce(
    logits: torch.Tensor, labels: torch.Tensor, weights: torch.Tensor | None = None, ignore_index: int = -1
) -> dict[str, torch.Tensor]:
    native_ok = logits.dtype in (torch.bfloat16, torch.float32) and labels.dtype == torch.int64 and use_native(logits, labels)
    if not native_ok:
        return semantic_ce_reference(logits, labels, weights, ignore_index)
    w = weights.float().contiguous() if weights is not None else None
    loss, stats, hist = _SemanticCE.apply(logits.contiguous(), labels.contiguous(), w, int(ignore_index))
    inter, pred, lab = hist[0], hist[1], hist[2]
    present = lab > 0
    union = (pred + lab - inter).clamp_min(1.0)
    n_present = present.sum()
    miou = torch.where(n_present > 0, ((inter / union) * present).sum() / n_present.clamp_min(1),
                       torch.full_like(n_present, float("nan"), dtype=torch.float64))
    return {
        "loss": loss,
        "pixel_accuracy": (stats[3] / stats[2].clamp_min(1.0)).float(),
        "mean_iou": miou.float(),
        "classes_present": n_present.float(),
    }


def connected_components(labels: torch.Tensor) -> torch.Tensor:
    """Host 6-connected components of equal positive ids -> int64, background / negatives kept."""
    return native().connected_components_cpu(labels.cpu())
