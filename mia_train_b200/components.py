"""Imports every concrete component so the registries are populated (reference `src/components.py:11-23`).

A registry decorator runs only when its module is imported. Adding a component means writing it and
adding one line here.
"""

from __future__ import annotations

from .algorithms import affinity_seg, dinov3_ssl, mae, muvit_mae, semantic_seg, simmim  # noqa: F401
from .data import huggingface, miao_dataset, synthetic  # noqa: F401
from .evals import semantic_seg as semantic_seg_eval  # noqa: F401
from .models import dinov3_vit, dinov3_vit3d, muvit, vit  # noqa: F401
