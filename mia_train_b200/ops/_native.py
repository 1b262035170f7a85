"""Loading of the in-tree sm_100a extension and the CUDA-vs-CPU dispatch rule.

Every op in `mia_train_b200.ops` runs this framework's own CUDA kernels when its inputs live on a
CUDA device, and plain PyTorch math on the CPU (the CPU path doubles as the numerical oracle in the
tests). There is no silent fallback on a GPU: if the extension cannot be loaded there, the op
raises.

`reference_math()` forces the PyTorch path everywhere for its duration. The engine uses it while
counting a step's FLOPs with `torch.utils.flop_counter`, which cannot see custom kernels.
"""

from __future__ import annotations

import contextlib
import importlib
import os
import threading
from collections.abc import Iterator
from pathlib import Path
from types import ModuleType

import torch

_EXT_NAME = "mia_train_b200._C"
_lock = threading.Lock()
_module: ModuleType | None = None
_load_error: str | None = None
_state = threading.local()

EXT_DIR = Path(__file__).resolve().parents[1]


def _try_load() -> ModuleType | None:
    global _module, _load_error
    with _lock:
        if _module is not None or _load_error is not None:
            return _module
        try:
            _module = importlib.import_module(_EXT_NAME)
        except Exception as error:  # noqa: BLE001 - the message is re-raised where it matters
            _load_error = f"{type(error).__name__}: {error}"
        return _module


def native_available() -> bool:
    return _try_load() is not None


def native() -> ModuleType:
    """The compiled extension; raises with the build hint when it is missing."""
    mod = _try_load()
    if mod is None:
        raise RuntimeError(
            f"the mia_train_b200 CUDA extension is not loadable ({_load_error}); build it with "
            "`python setup.py build_ext --inplace` (or __graft_entry__.build())"
        )
    return mod


def loaded_library_path() -> str | None:
    mod = _try_load()
    return getattr(mod, "__file__", None) if mod is not None else None


@contextlib.contextmanager
def reference_math() -> Iterator[None]:
    previous = getattr(_state, "force_torch", False)
    _state.force_torch = True
    try:
        yield
    finally:
        _state.force_torch = previous


def forcing_reference() -> bool:
    return bool(getattr(_state, "force_torch", False)) or os.environ.get("MIA_FORCE_TORCH_OPS") == "1"


def use_native(*tensors: torch.Tensor) -> bool:
    """True when the native kernels must run: CUDA inputs and no reference-math override."""
    if forcing_reference():
        return False
    if not any(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors):
        return False
    native()  # raises if missing: CUDA inputs never fall back silently
    return True
