"""Module-tree traversal that passes each module's dotted path to the callback.

Interface of reference `src/utils/module_ops.py:14-61` (the `named_apply(fn, module, name,
depth_first, include_root)` convention that DINOv3-style weight initialisers are written against:
the callback is called with `module=` and `name=` keywords). `nn.Module.apply` hands over only the
module, but initialisation here depends on where a module sits in the tree.

The traversal is an explicit stack rather than recursion, so arbitrarily deep trees are fine, and
`named_replace` swaps children through their parent's attribute.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator

import torch.nn as nn


def _join(prefix: str, child: str) -> str:
    return child if not prefix else prefix + "." + child


def _visit_order(root: nn.Module, root_name: str, post_order: bool) -> Iterator[tuple[str, nn.Module, nn.Module | None, str]]:
    """(dotted name, module, parent, attribute in parent) for every module under `root`, root first
    (pre-order) or children first (post-order)."""
    # stack entries: (name, module, parent, attribute, children already expanded)
    stack: list[tuple[str, nn.Module, nn.Module | None, str, bool]] = [(root_name, root, None, "", False)]
    while stack:
        name, module, parent, attr, expanded = stack.pop()
        if post_order and expanded:
            yield name, module, parent, attr
            continue
        if not post_order:
            yield name, module, parent, attr
        if post_order:
            stack.append((name, module, parent, attr, True))
        children = list(module.named_children())
        for child_attr, child in reversed(children):
            stack.append((_join(name, child_attr), child, module, child_attr, False))


def named_apply(
    fn: Callable[..., None],
    module: nn.Module,
    name: str = "",
    depth_first: bool = True,
    include_root: bool = False,
) -> nn.Module:
    """Call `fn(module=m, name=path)` for every module below `module` (and `module` itself when
    `include_root`). `depth_first` visits children before their parent."""
    for path, m, parent, _ in list(_visit_order(module, name, post_order=depth_first)):
        if parent is None and not include_root:
            continue
        fn(module=m, name=path)
    return module


def named_replace(
    fn: Callable[..., nn.Module],
    module: nn.Module,
    name: str = "",
    depth_first: bool = True,
    include_root: bool = False,
) -> nn.Module:
    """Like `named_apply`, but whatever `fn` returns takes the visited module's place in its parent
    (or becomes the returned root when `include_root`). Children first with `depth_first`; otherwise
    a parent is replaced first and the traversal continues into the replacement's children."""
    if depth_first:
        result = module
        for path, m, parent, attr in list(_visit_order(module, name, post_order=True)):
            if parent is None:
                if include_root:
                    result = fn(module=m, name=path)
            else:
                setattr(parent, attr, fn(module=m, name=path))
        return result
    root = fn(module=module, name=name) if include_root else module
    pending: list[tuple[str, nn.Module]] = [(name, root)]
    while pending:
        prefix, parent = pending.pop()
        for attr, child in list(parent.named_children()):
            path = _join(prefix, attr)
            replacement = fn(module=child, name=path)
            setattr(parent, attr, replacement)
            pending.append((path, replacement))
    return root
