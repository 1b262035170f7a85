"""Module-tree walks that hand the dotted name to the callback (reference
`src/utils/module_ops.py:14-61`). DINOv3's weight init depends on where a module sits, which
`nn.Module.apply` cannot express."""

from __future__ import annotations

from collections.abc import Callable

import torch.nn as nn


def named_apply(
    fn: Callable[..., None],
    module: nn.Module,
    name: str = "",
    depth_first: bool = True,
    include_root: bool = False,
) -> nn.Module:
    """Call `fn(module=..., name=...)` on every submodule."""
    if include_root and not depth_first:
        fn(module=module, name=name)
    for child_name, child in module.named_children():
        named_apply(fn, child, f"{name}.{child_name}" if name else child_name, depth_first, True)
    if include_root and depth_first:
        fn(module=module, name=name)
    return module


def named_replace(
    fn: Callable[..., nn.Module],
    module: nn.Module,
    name: str = "",
    depth_first: bool = True,
    include_root: bool = False,
) -> nn.Module:
    """Like `named_apply`, but the callback's return value replaces the module it was given."""
    if include_root and not depth_first:
        module = fn(module=module, name=name)
    for child_name, child in list(module.named_children()):
        full = f"{name}.{child_name}" if name else child_name
        setattr(module, child_name, named_replace(fn, child, full, depth_first, True))
    if include_root and depth_first:
        module = fn(module=module, name=name)
    return module
