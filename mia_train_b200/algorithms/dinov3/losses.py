"""DINOv3 losses: Sinkhorn-Knopp centring, DINO, iBOT and KoLeo (reference
`src/algorithms/dinov3/losses.py:48-206`).

* `sinkhorn_knopp(logits, T, n_iter)`: Q = exp(logits / T)^T in fp32, normalised by its global sum
  (all-reduced), then `n_iter` rounds of: rows summed globally (all-reduced) and divided by K,
  columns summed locally and divided by the global batch; finally scaled by the batch. The
  exponent is not clamped, as in the reference. On CUDA the same iterates run as two scaling
  vectors over native reductions (`_sinkhorn_native`): 2 n_iter + 2 passes over the logits
  instead of about ten full-matrix passes per iteration.
* `DINOLoss`: cross-entropy of the student's temperature-softened log-softmax against the teacher
  probabilities over all (student, teacher) view pairs, optionally ignoring same-view pairs.
* `IBOTPatchLoss`: the same on masked patches, each sample's patches weighted by 1 / its count; the
  global masked-patch count is all-reduced.
* `KoLeoLoss`: -mean log distance to the nearest neighbour of L2-normalised features, outside
  autocast.

On CUDA the DINO and iBOT cross-entropies run on one native soft-target cross-entropy kernel pair
(log-sum-exp and the teacher dot products in one pass over each student row; `ops/dino.py`) and
KoLeo on a one-CTA kernel pair; the PyTorch formulas above remain the CPU path and the oracles.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F


def _world_size() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _all_reduce(t: torch.Tensor) -> torch.Tensor:
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(t)
    return t


def _sinkhorn_native(logits: torch.Tensor, temperature: float, n_iterations: int, total: float,
                     colsum: torch.Tensor | None = None) -> torch.Tensor:
    """The iterates of `sinkhorn_knopp` as scaling vectors, P[b, k] = E[b, k] r[k] s[b] with
    E = exp(x / T): start r = 1, s = 1 / S0 (S0 = global sum of E); each iteration sets
    r[k] = 1 / (K A[k]) with A[k] = sum_b E[b, k] s[b] (all-reduced, as the reference's row sums)
    and s[b] = 1 / (B T[b]) with T[b] = sum_k E[b, k] r[k]; the result is E r s B. Native kernels
    (`csrc/sinkhorn.cu`) do the two reductions and the final write, recomputing E each pass."""
    from ...ops._native import native

    ext = native()
    x = logits.contiguous()
    b, k = x.shape
    a = torch.empty(k, device=x.device, dtype=torch.float32)
    t = torch.empty(b, device=x.device, dtype=torch.float32)
    if colsum is not None:  # sum_b E[b, k], already reduced by the prototype GEMM's epilogue
        a.copy_(colsum)
    else:
        ext.sinkhorn_colsum(x, float(temperature), None, a)  # sum_b E[b, k]
    _all_reduce(a)
    s0 = a.sum()
    r = torch.ones(k, device=x.device, dtype=torch.float32)
    s = torch.ones(b, device=x.device, dtype=torch.float32) / s0
    for it in range(n_iterations):
        if it == 0:
            r = s0 / (k * a)  # A = a / S0 with s = 1 / S0
        else:
            ext.sinkhorn_colsum(x, float(temperature), s, a)
            _all_reduce(a)
            r = 1.0 / (k * a)
        ext.sinkhorn_rowsum(x, float(temperature), r, t)
        s = 1.0 / (total * t)
    out = torch.empty(b, k, device=x.device, dtype=torch.float32)
    ext.sinkhorn_scale(x, float(temperature), r.contiguous(), (s * total).contiguous(), 1.0, out)
    return out


def sinkhorn_knopp(
    logits: torch.Tensor, temperature: float, n_iterations: int = 3, batch_size: float | None = None,
    colsum: torch.Tensor | None = None,
) -> torch.Tensor:
    """`colsum` (optional, this rank's sum_b exp(logits / T)) lets the native path skip its first pass."""
    from ...ops._native import use_native

    world = _world_size()
    total = float(logits.shape[0] * world) if batch_size is None else float(batch_size)
    # Below ~64 rows per rank the iteration is bound by launch overhead either way and PyTorch's is
    # shorter. The two paths issue different collectives, so the choice is made from the global
    # row count (the same on every rank), never from this rank's own, possibly uneven, share.
    if (use_native(logits) and logits.dim() == 2 and total >= 64 * world and logits.shape[1] % 8 == 0
            and logits.dtype in (torch.float32, torch.bfloat16)):
        return _sinkhorn_native(logits, temperature, n_iterations, total, colsum)
    q = torch.exp(logits.float() / temperature).t()  # (K, B_local)
    k = q.shape[0]
    q /= _all_reduce(torch.sum(q))
    for _ in range(n_iterations):
        q /= _all_reduce(torch.sum(q, dim=1, keepdim=True))
        q /= k
        q /= torch.sum(q, dim=0, keepdim=True)
        q /= total
    q *= total
    return q.t()


class DINOLoss(nn.Module):
    def __init__(self, out_dim: int, student_temp: float = 0.1) -> None:
        super().__init__()
        self.out_dim = out_dim
        self.student_temp = student_temp

    def sinkhorn_knopp_teacher(self, teacher_logits: torch.Tensor, teacher_temp: float, n_iterations: int = 3,
                               colsum: torch.Tensor | None = None):
        return sinkhorn_knopp(teacher_logits, teacher_temp, n_iterations, colsum=colsum)

    def forward(self, student_logits: torch.Tensor, teacher_probs: torch.Tensor, ignore_diagonal: bool = False):
        from ...ops._native import use_native

        if use_native(student_logits):
            return self._forward_native(student_logits, teacher_probs, ignore_diagonal)
        log_probs = F.log_softmax(student_logits.float() / self.student_temp, dim=-1)
        n_s, b, _ = log_probs.shape
        n_t = teacher_probs.shape[0]
        if not ignore_diagonal:
            return -torch.einsum("sbk,tbk->", log_probs, teacher_probs) / (b * n_s * n_t)
        pairwise = -torch.einsum("sbk,tbk->st", log_probs, teacher_probs)
        diag = min(n_s, n_t)
        pairwise = torch.diagonal_scatter(pairwise, torch.zeros(diag, device=pairwise.device, dtype=pairwise.dtype))
        return pairwise.sum() / (b * n_s * n_t - b * diag)


    def _forward_native(self, student_logits, teacher_probs, ignore_diagonal):
        """Student row (s, b) pairs with teacher rows (t, b); same-view pairs get weight 0 when ignored."""
        from ...ops.dino import soft_cross_entropy

        n_s, b, k = student_logits.shape
        n_t = teacher_probs.shape[0]
        dev = student_logits.device
        s_idx = torch.arange(n_s, device=dev).view(n_s, 1, 1)
        b_idx = torch.arange(b, device=dev).view(1, b, 1)
        t_idx = torch.arange(n_t, device=dev).view(1, 1, n_t)
        pairs = (t_idx * b + b_idx).expand(n_s, b, n_t).reshape(n_s * b, n_t)
        weights = torch.ones(n_s, b, n_t, device=dev)
        diag = min(n_s, n_t)
        norm = float(b * n_s * n_t)
        if ignore_diagonal:
            weights = weights * (s_idx != t_idx).float()
            norm = float(b * n_s * n_t - b * diag)
        return soft_cross_entropy(student_logits.reshape(n_s * b, k), teacher_probs.reshape(n_t * b, k), pairs,
                                  weights.reshape(n_s * b, n_t), self.student_temp, norm)


class IBOTPatchLoss(nn.Module):
    def __init__(self, patch_out_dim: int, student_temp: float = 0.1) -> None:
        super().__init__()
        self.patch_out_dim = patch_out_dim
        self.student_temp = student_temp

    def sinkhorn_knopp_teacher(self, teacher_logits, teacher_temp, n_masked_patches=None, n_iterations=3,
                               colsum=None):
        if n_masked_patches is None:
            n_masked_patches = teacher_logits.shape[0]
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            # the masked patch count of the whole data-parallel batch: one all-reduce and one read
            total = torch.full((), float(n_masked_patches), device=teacher_logits.device, dtype=torch.float32)
            _all_reduce(total)
            count = float(total.item())
        else:
            count = float(n_masked_patches)  # known on the host: no device round trip
        return sinkhorn_knopp(teacher_logits, teacher_temp, n_iterations, batch_size=count, colsum=colsum)

    def forward_masked(self, student_logits, teacher_probs, student_masks_flat, n_masked_patches=None,
                       masks_weight=None):
        from ...ops._native import use_native

        if masks_weight is None:
            masks_weight = (
                (1 / student_masks_flat.sum(-1).clamp(min=1.0)).unsqueeze(-1).expand_as(student_masks_flat)[student_masks_flat]
            )
        if use_native(student_logits) and student_logits.dim() == 2:
            from ...ops.dino import soft_cross_entropy

            rows = student_logits.shape[0]
            w = masks_weight.float().reshape(-1)[:rows]
            if w.shape[0] < rows:  # rows past the masked patches (padding) carry no loss
                w = torch.cat([w, w.new_zeros(rows - w.shape[0])])
            if n_masked_patches is not None:
                w = torch.where(torch.arange(rows, device=w.device) < n_masked_patches, w, torch.zeros_like(w))
            pairs = torch.arange(rows, device=student_logits.device, dtype=torch.int32).view(rows, 1)
            return soft_cross_entropy(student_logits, teacher_probs, pairs, w.view(rows, 1), self.student_temp,
                                      float(student_masks_flat.shape[0]))
        loss = torch.sum(teacher_probs * F.log_softmax(student_logits.float() / self.student_temp, dim=-1), dim=-1)
        if n_masked_patches is not None:
            loss = loss[:n_masked_patches]
        return -(loss * masks_weight).sum() / student_masks_flat.shape[0]


class KoLeoLoss(nn.Module):
    def __init__(self, eps: float = 1e-8) -> None:
        super().__init__()
        self.eps = eps
        self.pdist = nn.PairwiseDistance(2, eps=eps)

    def _pairwise_nearest(self, x: torch.Tensor) -> torch.Tensor:
        dots = torch.mm(x, x.t())
        n = x.shape[0]
        dots.view(-1)[:: n + 1].fill_(-1)
        return torch.argmax(dots, dim=1)

    def forward(self, student_output: torch.Tensor) -> torch.Tensor:
        from ...ops._native import use_native

        if use_native(student_output):
            from ...ops.dino import koleo

            with torch.autocast("cuda", enabled=False):
                return koleo(student_output, self.eps)
        with torch.autocast("cuda", enabled=False), torch.autocast("cpu", enabled=False):
            x = F.normalize(student_output.float(), eps=self.eps, p=2, dim=-1)
            nearest = self._pairwise_nearest(x)
            return -torch.log(self.pdist(x, x[nearest]) + self.eps).mean()
