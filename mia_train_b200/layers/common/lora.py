"""LoRA by in-place class promotion (reference `src/layers/common/lora.py:39-162`).

`promote(linear, rank, alpha)` turns an `nn.Linear` into `LoRA<Base>` in place: parameter names
are unchanged and `lora_a` (rank, in; kaiming-uniform), `lora_b` (out, rank; zeros) and a
persistent `lora_scaling` buffer (alpha / rank) are added, so the adapted layer starts exactly equal
to the base. `merge_lora()` folds the delta into the weight and reverts the class.

`apply_linear(module, x, ...)` is how every layer here calls a projection: it runs the native
fused-epilogue GEMM on the base weight and, for an adapted module, adds the low-rank delta
`(x A^T) B^T * scaling` (two rank-r GEMMs).
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ...ops.linear import linear


class LoRAMixin:
    in_features: int
    out_features: int
    weight: nn.Parameter

    def init_lora(self, rank: int, alpha: float) -> None:
        if rank < 1:
            raise ValueError(f"LoRA rank must be >= 1, got {rank}")
        self.lora_rank = rank
        opts = {"device": self.weight.device, "dtype": self.weight.dtype}
        self.lora_a = nn.Parameter(torch.empty(rank, self.in_features, **opts))
        self.lora_b = nn.Parameter(torch.zeros(self.out_features, rank, **opts))
        self.register_buffer("lora_scaling", torch.tensor(alpha / rank, **opts), persistent=True)  # type: ignore[attr-defined]
        self.reset_lora_parameters()

    def reset_lora_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.lora_a, a=math.sqrt(5))
        nn.init.zeros_(self.lora_b)

    def lora_delta(self) -> torch.Tensor:
        return self.lora_scaling * (self.lora_b @ self.lora_a)

    def lora_forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(F.linear(x, self.lora_a), self.lora_b) * self.lora_scaling

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        return super().forward(input) + self.lora_forward(input)  # type: ignore[misc]

    @torch.no_grad()
    def merge_lora(self) -> None:
        self.weight.add_(self.lora_delta().to(self.weight.dtype))
        del self.lora_a
        del self.lora_b
        del self.lora_rank
        del self.lora_scaling
        self.__class__ = type(self).__bases__[1]


_PROMOTED: dict[type, type] = {}


def promote(module: nn.Linear, *, rank: int, alpha: float) -> nn.Linear:
    if isinstance(module, LoRAMixin):
        raise ValueError(f"{type(module).__name__} is already adapted; promoting twice would double the delta")
    if not isinstance(module, nn.Linear):
        raise TypeError(f"LoRA adapts nn.Linear layers; got {type(module).__name__}")
    base = type(module)
    if base not in _PROMOTED:
        _PROMOTED[base] = type(f"LoRA{base.__name__}", (LoRAMixin, base), {})
    module.__class__ = _PROMOTED[base]
    module.init_lora(rank, alpha)  # type: ignore[attr-defined]
    return module


def adapted_modules(root: nn.Module) -> list[tuple[str, LoRAMixin]]:
    return [(name, m) for name, m in root.named_modules() if isinstance(m, LoRAMixin)]


def merge_all(root: nn.Module) -> list[str]:
    merged = []
    for name, module in adapted_modules(root):
        module.merge_lora()
        merged.append(name)
    return merged


_OWN_BIAS = object()


def apply_linear(
    module: nn.Linear,
    x: torch.Tensor,
    activation: str | None = None,
    residual: torch.Tensor | None = None,
    gamma: torch.Tensor | None = None,
    bias: Any = _OWN_BIAS,
) -> torch.Tensor:
    """`residual + gamma * act(module(x))` with the epilogue fused into the native GEMM; `bias`
    replaces the module's own bias (a masked-key-bias qkv passes its masked bias), adapter included."""
    b = module.bias if bias is _OWN_BIAS else bias
    if hasattr(module, "_tp_mode"):  # a tensor-parallel shard: local GEMM plus its collective
        from ...parallel.tensor_parallel import tp_linear

        extra = {} if bias is _OWN_BIAS else {"bias": b}
        return tp_linear(module, x, activation=activation, residual=residual, gamma=gamma, **extra)
    if isinstance(module, LoRAMixin):
        if gamma is None:
            from ...ops.linear import lora_linear

            fused = lora_linear(x, module.weight, b, module.lora_a, module.lora_b,
                                float(module.lora_scaling), activation=activation, residual=residual)
            if fused is not None:
                return fused
        y = linear(x, module.weight, b)
        y = y + module.lora_forward(x).to(y.dtype)
        if activation == "gelu":
            y = F.gelu(y)
        if gamma is not None:
            y = y * gamma
        return y if residual is None else residual + y
    return linear(x, module.weight, b, activation=activation, residual=residual, gamma=gamma)


def is_adapted(module: nn.Module) -> bool:
    return isinstance(module, LoRAMixin)


def needs_per_layer(module: nn.Module) -> bool:
    """LoRA-adapted or tensor-parallel: the layer must run through `apply_linear`, not a fused op."""
    return isinstance(module, LoRAMixin) or hasattr(module, "_tp_mode")
