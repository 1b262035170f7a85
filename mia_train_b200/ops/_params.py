"""Parameter-side conventions shared by the native ops.

* A parameter may carry `_mia_shadow`: a bf16 copy kept current by the fused optimizer. GEMMs read
  it instead of casting the fp32 weight on every call.
* A parameter may carry `main_grad`: a preallocated fp32 buffer (a view into a flat gradient
  buffer). Native backward kernels then accumulate their weight gradient straight into it (GEMM
  epilogue `accumulate`, column-sum `accumulate`, norm kernels' atomics) and return no autograd
  gradient for the parameter, so no separate gradient tensor is ever materialised or added.
"""

from __future__ import annotations

import torch


def compute_weight(weight: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    shadow = getattr(weight, "_mia_shadow", None)
    if shadow is not None and shadow.dtype == dtype:
        return shadow
    return weight.to(dtype)


def grad_sink(param: torch.Tensor | None) -> torch.Tensor | None:
    if param is None or not param.requires_grad:
        return None
    return getattr(param, "main_grad", None)
