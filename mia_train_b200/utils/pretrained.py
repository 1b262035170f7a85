"""`[init]`: start a run from weights trained elsewhere.

Interface of reference `src/utils/pretrained.py:38-395` (the `[init]` keys and what they mean);
the implementation is this framework's own. Loading is a short pipeline over a flat
name -> tensor mapping:

1. `read_state_dict` -- a `.pth` / `.pt` file, or a DCP checkpoint directory converted through
   `dcp_to_torch_save`; a wrapper dict (`model`, `state_dict`, `teacher`, `student`) is opened.
2. prefix selection -- keep the keys under `prefix`, with the prefix removed.
3. LoRA folding (`merge_lora`) -- W <- W + s * B @ A for every adapter in the checkpoint.
4. matching -- each model tensor takes the checkpoint tensor of the same name: copied when shapes
   agree, inflated from a 2-D kernel to a 3-D one when `inflate` is set, otherwise a mismatch.
5. verdict -- in strict mode a mismatch, a load that matched nothing, or checkpoint tensors nobody
   took (unless `allow_unused`) raise, with a hint about the configuration difference that usually
   causes them.
"""

from __future__ import annotations

import logging
import tempfile
from collections.abc import Iterable, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

logger = logging.getLogger(__name__)

# Wrapper keys that checkpoints from other trainers put around the weights, in lookup order.
NESTING_KEYS = ("model", "state_dict", "teacher", "student")


@dataclass
class LoadReport:
    """What happened to every tensor of the model and of the checkpoint."""

    copied: list[str] = field(default_factory=list)
    inflated: list[str] = field(default_factory=list)
    merged: list[str] = field(default_factory=list)
    skipped: list[str] = field(default_factory=list)
    kept_initial: list[str] = field(default_factory=list)
    unused: list[str] = field(default_factory=list)
    mismatched: list[tuple[str, tuple[int, ...], tuple[int, ...]]] = field(default_factory=list)
    filtered_by_prefix: list[str] = field(default_factory=list)

    def counts(self) -> dict[str, int]:
        return {
            "copied": len(self.copied),
            "inflated 2D->3D": len(self.inflated),
            "LoRA adapters merged": len(self.merged),
            "skipped": len(self.skipped),
            "kept at initial value": len(self.kept_initial),
            "unused from checkpoint": len(self.unused),
            "shape mismatches": len(self.mismatched),
            "filtered out by prefix": len(self.filtered_by_prefix),
        }

    def summary(self) -> str:
        always = {"copied", "inflated 2D->3D", "LoRA adapters merged", "skipped", "kept at initial value",
                  "unused from checkpoint"}
        return ", ".join(f"{n} {label}" for label, n in self.counts().items() if n or label in always)


# ---------------------------------------------------------------------------------------- reading
def _tensors_of(mapping: dict[str, Any]) -> dict[str, torch.Tensor]:
    return {k: v for k, v in mapping.items() if isinstance(v, torch.Tensor)}


def _open_wrapper(obj: Any) -> dict[str, torch.Tensor]:
    if not isinstance(obj, dict):
        raise ValueError(f"expected a state dict, but the checkpoint holds a {type(obj).__name__}")
    nested = (obj.get(k) for k in NESTING_KEYS)
    for inner in nested:
        if isinstance(inner, dict) and _tensors_of(inner):
            return _tensors_of(inner)
    own = _tensors_of(obj)
    if own:
        return own
    raise ValueError(f"the checkpoint has no tensors, neither at its top level nor under {', '.join(NESTING_KEYS)}")


def read_state_dict(path: str | Path) -> dict[str, torch.Tensor]:
    """Name -> tensor (on the CPU) from a torch save file or a DCP directory."""
    where = Path(path)
    if where.is_dir():
        from torch.distributed.checkpoint.format_utils import dcp_to_torch_save

        with tempfile.TemporaryDirectory() as tmp:
            single = Path(tmp) / "single_file.pt"
            dcp_to_torch_save(str(where), str(single))
            return _open_wrapper(torch.load(single, map_location="cpu", weights_only=False))
    if not where.is_file():
        raise FileNotFoundError(f"[init] path {where} does not exist")
    return _open_wrapper(torch.load(where, map_location="cpu", weights_only=False))


# ------------------------------------------------------------------------------------ transforms
def inflate_2d_to_3d(weight: torch.Tensor, target: torch.Size) -> torch.Tensor:
    """A (O, I, h, w) kernel as a (O, I', d, h, w) one whose response to a volume that is constant
    along depth equals the 2-D kernel's response to one slice: every depth tap gets weight / d.
    Input channels are averaged down to one, or spread evenly from one."""
    if weight.dim() != 4 or len(target) != 5:
        raise ValueError(f"inflation takes a 4-D kernel to a 5-D one; got {tuple(weight.shape)} and {tuple(target)}")
    o, i, h, w = weight.shape
    to, ti, d, th, tw = target
    if (o, h, w) != (to, th, tw):
        raise ValueError(f"kernel {tuple(weight.shape)} cannot become {tuple(target)}: the output channels and "
                         "the in-plane size have to agree already")
    if i != ti:
        if ti == 1:
            weight = weight.mean(1, keepdim=True)
        elif i == 1:
            weight = weight.repeat(1, ti, 1, 1) / ti
        else:
            raise ValueError(f"no rule maps {i} input channels onto {ti}")
    return (weight[:, :, None] / d).repeat(1, 1, d, 1, 1).contiguous()


def merge_lora_tensors(checkpoint: dict[str, torch.Tensor]) -> tuple[dict[str, torch.Tensor], list[str]]:
    """Fold every `<layer>.lora_a/.lora_b/.lora_scaling` triple into `<layer>.weight`."""
    layers = sorted(k[: -len(".lora_a")] for k in checkpoint if k.endswith(".lora_a"))
    out = dict(checkpoint)
    for layer in layers:
        parts = {s: f"{layer}.{s}" for s in ("lora_a", "lora_b", "lora_scaling", "weight")}
        absent = [name for name in parts.values() if name not in out]
        if absent:
            raise ValueError(f"adapter {layer!r} cannot be folded: {', '.join(absent)} not in the checkpoint")
        w = out[parts["weight"]]
        a, b, s = (out.pop(parts[key]).to(w.dtype) for key in ("lora_a", "lora_b", "lora_scaling"))
        out[parts["weight"]] = torch.addmm(w, b, a, alpha=float(s)) if s.numel() == 1 else w + s * (b @ a)
    return out, layers


# ----------------------------------------------------------------------------------------- hints
_UNUSED_HINTS = (
    (("ls1.gamma", "ls2.gamma"), "layerscale_init (the released DINOv3 ViTs use 1.0e-05)"),
    (("bias_mask",), "mask_k_bias = true"),
    (("storage_tokens",), "n_storage_tokens (the released DINOv3 ViTs use 4)"),
)


def _hint_for_unused(names: Iterable[str]) -> str:
    names = list(names)
    wanted = [fix for needles, fix in _UNUSED_HINTS if any(n in key for key in names for n in needles)]
    if wanted:
        return "The checkpoint has parts this model was configured without; consider " + "; ".join(wanted) + "."
    return "If the extra tensors are expected, set allow_unused = true (or select a sub-tree with prefix)."


def _hint_for_mismatch(names: Iterable[str]) -> str:
    names = list(names)
    if any("rope_embed" in n for n in names):
        return ("RoPE period buffers depend on the model's own settings (and on 2-D vs 3-D); "
                'leave them at their initial values with skip = ["rope_embed."].')
    if any(n.startswith("patch_embed.") for n in names):
        return "A 2-D patch embedding needs inflate_2d_to_3d = true and the checkpoint's patch size."
    return "Compare embed_dim, depth, num_heads and patch_size with the checkpoint's."


# ---------------------------------------------------------------------------------------- loading
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
    """Copy matching tensors of the checkpoint at `path` into `model` (see the module docstring)."""
    source = read_state_dict(path)
    report = LoadReport()
    if prefix:
        report.filtered_by_prefix = sorted(k for k in source if not k.startswith(prefix))
        source = {k.removeprefix(prefix): v for k, v in source.items() if k.startswith(prefix)}
    if merge_lora:
        source, report.merged = merge_lora_tensors(source)
        if not report.merged:
            raise ValueError(f"merge_lora = true, but {path} contains no LoRA adapter to fold")

    def skipped(name: str) -> bool:
        return any(name.startswith(s) for s in skip)

    destinations = {**dict(model.named_parameters()), **dict(model.named_buffers())}
    remaining = dict(source)
    with torch.no_grad():
        for name, dest in destinations.items():
            src = remaining.pop(name, None)
            if skipped(name):
                report.skipped.append(name)
            elif src is None:
                report.kept_initial.append(name)
            elif src.shape == dest.shape:
                dest.copy_(src)
                report.copied.append(name)
            elif inflate and src.dim() == 4 and dest.dim() == 5:
                dest.copy_(inflate_2d_to_3d(src, dest.shape))
                report.inflated.append(name)
            else:
                report.mismatched.append((name, tuple(src.shape), tuple(dest.shape)))
    report.unused = sorted(k for k in remaining if not skipped(k))
    logger.info("[init] %s <- %s: %s", type(model).__name__, path, report.summary())
    if strict:
        _enforce(report, path, remaining, destinations, allow_unused)
    _announce(model, Path(path), report)
    return report


def _enforce(report: LoadReport, path: Any, remaining: dict, destinations: dict, allow_unused: bool) -> None:
    if report.mismatched:
        rows = "\n".join(f"  {name}: checkpoint {src} vs model {dst}" for name, src, dst in report.mismatched)
        raise ValueError(f"[init] shapes differ for {len(report.mismatched)} tensor(s) of {path}:\n{rows}\n"
                         + _hint_for_mismatch(n for n, _, _ in report.mismatched))
    if not (report.copied or report.inflated):
        raise ValueError(
            f"[init] no tensor of {path} fits this model: the checkpoint has e.g. {sorted(remaining)[:5]}, the model "
            f"e.g. {sorted(destinations)[:5]} (if the weights sit under a sub-tree, set prefix)"
        )
    if report.unused and not allow_unused:
        shown = ", ".join(report.unused[:6]) + (", ..." if len(report.unused) > 6 else "")
        raise ValueError(f"[init] {len(report.unused)} tensor(s) of {path} found no home in this model ({shown}). "
                         + _hint_for_unused(report.unused))


def _announce(model: nn.Module, path: Path, report: LoadReport) -> None:
    if dist.is_initialized() and dist.get_rank() != 0:
        return
    lines = [f"[init] {type(model).__name__} <- {path}", f"[init]   {report.summary()}"]
    for label, names in (("filtered out by prefix", report.filtered_by_prefix), ("skipped", report.skipped),
                         ("kept at initial value", report.kept_initial), ("unused from checkpoint", report.unused)):
        if names:
            lines.append(f"[init]   {len(names)} {label}: {', '.join(names[:4])}{' ...' if len(names) > 4 else ''}")
    print("\n".join(lines), flush=True)
