"""Imports every concrete component so the registries are populated (reference `src/components.py`).

A registry decorator runs only when its module is imported. Adding a component means writing it and
adding one line here.
"""

from __future__ import annotations

from .algorithms import mae  # noqa: F401
from .data import synthetic  # noqa: F401
from .models import vit  # noqa: F401
