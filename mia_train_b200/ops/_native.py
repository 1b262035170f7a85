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


# Codes a kernel writes to the per-device error word when a bounded wait runs out (common.cuh).
ERROR_CODES = {
    101: "GEMM TMA producer wait",
    102: "GEMM MMA issuer wait",
    103: "GEMM epilogue wait",
    201: "attention barrier wait",
    301: "collective flag wait",
    401: "sharded-optimizer reduce-scatter barrier",
    402: "sharded-optimizer gradient-norm exchange",
    403: "sharded-optimizer all-gather barrier",
    501: "symmetric-memory barrier",
    502: "tensor-parallel chunk flag wait",
    503: "tensor-parallel slot reuse wait",
}


class DeviceWaitError(RuntimeError):
    """A kernel gave up a bounded wait (a peer or a pipeline stage never arrived)."""

    def __init__(self, code: int, device: int) -> None:
        self.code = code
        self.device = device
        what = ERROR_CODES.get(code, "unknown wait")
        super().__init__(
            f"device {device}: a kernel abandoned a bounded wait ({what}, code {code}); the step's results "
            "are not trustworthy (a peer rank may be gone)"
        )


def device_error_code(device: int) -> int:
    """Read and clear the error word of `device` (synchronises with that device)."""
    return int(native().check_errors(int(device)))


def raise_on_device_errors(device: torch.device | int) -> None:
    """Raise `DeviceWaitError` if any kernel on `device` recorded a wait timeout since the last check.

    A no-op for CPU devices and when the extension is not loadable (no native kernel ran then).
    """
    if isinstance(device, torch.device):
        if device.type != "cuda":
            return
        index = device.index if device.index is not None else torch.cuda.current_device()
    else:
        index = int(device)
    if not native_available():
        return
    code = device_error_code(index)
    if code != 0:
        raise DeviceWaitError(code, index)
