"""`[init]`: start a run from weights trained elsewhere (reference `src/utils/pretrained.py:38-395`).

Reads a `.pth`/`.pt` state dict or a DCP directory (converted through `dcp_to_torch_save`),
unwraps it from `model` / `state_dict` / `teacher` / `student` nesting, keeps only keys under
`prefix` (stripped), optionally folds LoRA adapters into their weights, then copies every tensor
whose name and shape match, inflating 4-D conv kernels to 5-D (in-plane kernel replicated over
depth and divided by it; input channels averaged to one or spread from one) when asked. Strict mode
refuses shape mismatches, loads that matched nothing, and unused checkpoint tensors, each with a
hint naming the likely configuration difference.
"""

from __future__ import annotations

import logging
import tempfile
from collections.abc import Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

logger = logging.getLogger(__name__)
NESTING_KEYS = ("model", "state_dict", "teacher", "student")


@dataclass
class LoadReport:
    copied: list[str] = field(default_factory=list)
    inflated: list[str] = field(default_factory=list)
    merged: list[str] = field(default_factory=list)
    skipped: list[str] = field(default_factory=list)
    kept_initial: list[str] = field(default_factory=list)
    unused: list[str] = field(default_factory=list)
    mismatched: list[tuple[str, tuple[int, ...], tuple[int, ...]]] = field(default_factory=list)
    filtered_by_prefix: list[str] = field(default_factory=list)

    def summary(self) -> str:
        parts = [
            f"{len(self.copied)} copied",
            f"{len(self.inflated)} inflated 2D->3D",
            f"{len(self.merged)} LoRA adapters merged",
            f"{len(self.skipped)} skipped",
            f"{len(self.kept_initial)} kept at initial value",
            f"{len(self.unused)} unused from checkpoint",
        ]
        if self.mismatched:
            parts.append(f"{len(self.mismatched)} shape mismatches")
        if self.filtered_by_prefix:
            parts.append(f"{len(self.filtered_by_prefix)} filtered out by prefix")
        return ", ".join(parts)


def _unwrap(state: Any) -> dict[str, torch.Tensor]:
    if not isinstance(state, dict):
        raise ValueError(f"checkpoint is a {type(state).__name__}, not a state dict")
    for key in NESTING_KEYS:
        inner = state.get(key)
        if isinstance(inner, dict) and any(isinstance(v, torch.Tensor) for v in inner.values()):
            return {k: v for k, v in inner.items() if isinstance(v, torch.Tensor)}
    tensors = {k: v for k, v in state.items() if isinstance(v, torch.Tensor)}
    if not tensors:
        raise ValueError(f"checkpoint holds no tensors at the top level or under any of {list(NESTING_KEYS)}")
    return tensors


def read_state_dict(path: str | Path) -> dict[str, torch.Tensor]:
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(f"no checkpoint at {path}")
    if path.is_dir():
        from torch.distributed.checkpoint.format_utils import dcp_to_torch_save

        with tempfile.TemporaryDirectory() as scratch:
            flat = Path(scratch) / "converted.pt"
            dcp_to_torch_save(str(path), str(flat))
            return _unwrap(torch.load(flat, map_location="cpu", weights_only=False))
    return _unwrap(torch.load(path, map_location="cpu", weights_only=False))


def inflate_2d_to_3d(weight: torch.Tensor, target: torch.Size) -> torch.Tensor:
    if weight.ndim != 4 or len(target) != 5:
        raise ValueError(f"inflation maps a 4D kernel to a 5D one, got {tuple(weight.shape)} -> {tuple(target)}")
    out_c, in_c, h, w = weight.shape
    t_out, t_in, depth, t_h, t_w = target
    if (out_c, h, w) != (t_out, t_h, t_w):
        raise ValueError(
            f"cannot inflate a {tuple(weight.shape)} kernel into {tuple(target)}: output channels and the "
            "in-plane kernel must already match"
        )
    if in_c != t_in:
        if t_in == 1:
            weight = weight.mean(dim=1, keepdim=True)
        elif in_c == 1:
            weight = weight.expand(-1, t_in, -1, -1) / t_in
        else:
            raise ValueError(f"cannot map {in_c} checkpoint input channels onto {t_in}")
    return (weight.unsqueeze(2).expand(-1, -1, depth, -1, -1) / depth).contiguous()


def merge_lora_tensors(checkpoint: dict[str, torch.Tensor]) -> tuple[dict[str, torch.Tensor], list[str]]:
    out = dict(checkpoint)
    folded = []
    for key in sorted(checkpoint):
        if not key.endswith(".lora_a"):
            continue
        layer = key[: -len(".lora_a")]
        needed = [f"{layer}.{s}" for s in ("lora_a", "lora_b", "lora_scaling", "weight")]
        missing = [n for n in needed if n not in out]
        if missing:
            raise ValueError(f"cannot merge the LoRA adapter at {layer!r}: the checkpoint is missing {missing}")
        a = out.pop(f"{layer}.lora_a")
        b = out.pop(f"{layer}.lora_b")
        s = out.pop(f"{layer}.lora_scaling")
        base = out[f"{layer}.weight"]
        out[f"{layer}.weight"] = base + s.to(base.dtype) * (b.to(base.dtype) @ a.to(base.dtype))
        folded.append(layer)
    return out, folded


def load_pretrained(
    model: nn.Module,
    path: str | Path,
    *,
    prefix: str = "",
    inflate: bool = False,
    skip: Sequence[str] = (),
    strict: bool = True,
    allow_unused: bool = False,
    merge_lora: bool = False,
) -> LoadReport:
    checkpoint = read_state_dict(path)
    filtered: list[str] = []
    if prefix:
        filtered = sorted(k for k in checkpoint if not k.startswith(prefix))
        checkpoint = {k[len(prefix):]: v for k, v in checkpoint.items() if k.startswith(prefix)}
    merged: list[str] = []
    if merge_lora:
        checkpoint, merged = merge_lora_tensors(checkpoint)
        if not merged:
            raise ValueError(f"merge_lora is set but {path} holds no LoRA adapter, so nothing would be merged")
    targets: dict[str, torch.Tensor] = dict(model.named_parameters())
    targets.update(model.named_buffers())
    report = LoadReport(merged=merged, filtered_by_prefix=filtered)
    with torch.no_grad():
        for name, dest in targets.items():
            src = checkpoint.pop(name, None)
            if any(name.startswith(s) for s in skip):
                report.skipped.append(name)
                continue
            if src is None:
                report.kept_initial.append(name)
            elif src.shape == dest.shape:
                dest.copy_(src)
                report.copied.append(name)
            elif inflate and src.ndim == 4 and dest.ndim == 5:
                dest.copy_(inflate_2d_to_3d(src, dest.shape).to(dest.dtype))
                report.inflated.append(name)
            else:
                report.mismatched.append((name, tuple(src.shape), tuple(dest.shape)))
    report.unused = sorted(k for k in checkpoint if not any(k.startswith(s) for s in skip))
    logger.info("loaded pretrained weights from %s: %s", path, report.summary())
    if not strict:
        return report
    if report.mismatched:
        details = "\n".join(f"  {n}: checkpoint {s} vs model {d}" for n, s, d in report.mismatched)
        raise ValueError(f"{len(report.mismatched)} tensor(s) in {path} do not fit this model:\n{details}\n{_mismatch_hint(report)}")
    if not report.copied and not report.inflated:
        raise ValueError(
            f"nothing in {path} matched this model's parameters; the checkpoint offers keys like "
            f"{sorted(checkpoint)[:5]}, the model wants {sorted(targets)[:5]}. Set `prefix` if the "
            "checkpoint stores the encoder under one."
        )
    if report.unused and not allow_unused:
        more = " ..." if len(report.unused) > 6 else ""
        raise ValueError(
            f"{len(report.unused)} tensor(s) in {path} have no home in this model: {report.unused[:6]}{more}\n"
            f"{_unused_hint(report)}"
        )
    _log_load(model, Path(path), report)
    return report


def _log_load(model: nn.Module, path: Path, report: LoadReport) -> None:
    if dist.is_initialized() and dist.get_rank() != 0:
        return
    print(f"[init] {type(model).__name__} <- {path}", flush=True)
    print(f"[init]   {report.summary()}", flush=True)
    for label, names in (
        ("filtered out by prefix", report.filtered_by_prefix),
        ("skipped", report.skipped),
        ("kept at initial value", report.kept_initial),
        ("unused from checkpoint", report.unused),
    ):
        if names:
            more = " ..." if len(names) > 4 else ""
            print(f"[init]   {len(names)} {label}: {', '.join(names[:4])}{more}", flush=True)


def _unused_hint(report: LoadReport) -> str:
    missing = []
    if any("ls1.gamma" in k or "ls2.gamma" in k for k in report.unused):
        missing.append("layerscale_init (the released DINOv3 ViTs use 1.0e-05)")
    if any("bias_mask" in k for k in report.unused):
        missing.append("mask_k_bias = true")
    if any("storage_tokens" in k for k in report.unused):
        missing.append("n_storage_tokens (the released DINOv3 ViTs use 4)")
    if missing:
        return "The model appears to be missing: " + "; ".join(missing) + "."
    return "Set allow_unused = true if the checkpoint is expected to hold more than this model needs, or `prefix`."


def _mismatch_hint(report: LoadReport) -> str:
    for name, _, _ in report.mismatched:
        if "rope_embed" in name:
            return (
                "rope_embed buffers are derived from the model's own base and differ between 2D and 3D; "
                'add skip = ["rope_embed."] to [init]'
            )
        if name.startswith("patch_embed."):
            return "Set inflate_2d_to_3d = true and configure the model with the checkpoint's patch size."
    return "Check that embed_dim, depth, num_heads and patch_size match the checkpoint's."
