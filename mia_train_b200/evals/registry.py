"""`EvalRegistry`: name -> evaluation task (reference `src/evals/registry.py`)."""

from __future__ import annotations

from ..utils.registry import Registry
from .base import BaseEvalTask

EvalRegistry: Registry[BaseEvalTask] = Registry(BaseEvalTask, kind="eval task")
