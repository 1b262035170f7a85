"""`FusedAdamW`: torch.optim.AdamW semantics on one native multi-tensor kernel.

Same update rule as `torch.optim.AdamW` (decoupled weight decay, bias-corrected moments, eps added
to the corrected root), the same per-parameter state keys (`step`, `exp_avg`, `exp_avg_sq`) so DCP
checkpoints interchange with the stock optimizer, and the same param-group fields (`lr`,
`weight_decay`, `betas`, `eps`) so `WarmupDecaySchedule` drives it unchanged.

Per step it issues one host->device copy of the per-group (lr, weight_decay, beta1, beta2) table
and one kernel launch over every parameter; `step` counters live on the device. An optional
device-side `grad_scale` (the grad-clip coefficient) is applied as gradients are read. Parameters
whose grad is None are skipped, and their step does not advance, as in torch. A parameter with a
`main_grad` buffer (see `ops/_params.py`) is updated from it, and one with a `_mia_shadow` bf16
copy gets that copy rewritten by the same kernel.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.optim import Optimizer

from ..ops.optim import adamw_step


class FusedAdamW(Optimizer):
    def __init__(
        self,
        params: Any,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
    ) -> None:
        defaults = {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay}
        super().__init__(params, defaults)
        self._hyper_host: torch.Tensor | None = None
        self._hyper_dev: torch.Tensor | None = None
        self.grad_scale: torch.Tensor | None = None

    def _init_state(self, p: torch.Tensor) -> dict[str, Any]:
        state = self.state[p]
        if len(state) == 0:
            state["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        elif state["step"].device != p.device:
            state["step"] = state["step"].to(p.device, torch.float32)
        return state

    def _hyper(self, device: torch.device) -> torch.Tensor:
        external = getattr(self, "external_hyper", None)
        if external is not None:  # a device-side schedule (see engine/graph_step.py)
            return external
        g = len(self.param_groups)
        if self._hyper_host is None or self._hyper_host.shape[0] != g:
            self._hyper_host = torch.empty((g, 4), dtype=torch.float32, pin_memory=torch.cuda.is_available())
            self._hyper_dev = torch.empty((g, 4), dtype=torch.float32, device=device)
        for i, group in enumerate(self.param_groups):
            b1, b2 = group["betas"]
            self._hyper_host[i, 0] = float(group["lr"])
            self._hyper_host[i, 1] = float(group["weight_decay"])
            self._hyper_host[i, 2] = float(b1)
            self._hyper_host[i, 3] = float(b2)
        assert self._hyper_dev is not None
        self._hyper_dev.copy_(self._hyper_host, non_blocking=True)
        return self._hyper_dev

    @torch.no_grad()
    def step(self, closure: Any = None) -> Any:  # type: ignore[override]
        loss = closure() if closure is not None else None
        params, grads, m, v, steps, gidx, shadows = [], [], [], [], [], [], []
        eps = None
        have_shadow = False
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                grad = p.grad if p.grad is not None else getattr(p, "main_grad", None)
                if grad is None:
                    continue
                if grad.is_sparse:
                    raise RuntimeError("FusedAdamW does not support sparse gradients")
                state = self._init_state(p)
                params.append(p)
                grads.append(grad)
                shadow = getattr(p, "_mia_shadow", None)
                have_shadow = have_shadow or shadow is not None
                shadows.append(shadow if shadow is not None else self._empty(p.device))
                m.append(state["exp_avg"])
                v.append(state["exp_avg_sq"])
                steps.append(state["step"])
                gidx.append(gi)
                eps = group["eps"] if eps is None else eps
                if group["eps"] != eps:
                    raise ValueError("FusedAdamW needs one eps for all param groups")
        if not params:
            return loss
        device = params[0].device
        hyper = self._hyper(device)
        key = tuple(gidx)
        cached = getattr(self, "_gidx_cache", None)
        if cached is None or cached[0] != key:
            self._gidx_cache = (key, torch.tensor(gidx, dtype=torch.int32, device=device))
        adamw_step(
            params, grads, m, v, steps, self._gidx_cache[1], hyper, float(eps), self.grad_scale,
            shadows if have_shadow else None,
        )
        return loss

    def _empty(self, device: torch.device) -> torch.Tensor:
        cache = self.__dict__.setdefault("_empty_cache", {})
        if device not in cache:
            cache[device] = torch.empty(0, device=device, dtype=torch.bfloat16)
        return cache[device]
