"""Name -> class registries that let a TOML config select a component by name.

Behaviour follows the reference's `src/utils/registry.py:9-42`: a duplicate name or a class that is
not a subclass of the registry's base is refused at registration time, and an unknown name lists
what is available.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any, Generic, TypeVar

T = TypeVar("T")


class Registry(Generic[T]):
    """Maps names to subclasses of one base class."""

    def __init__(self, base: type[Any], kind: str = "component") -> None:
        self._base = base
        self._kind = kind
        self._entries: dict[str, type[T]] = {}

    def register(self, name: str) -> Callable[[type[T]], type[T]]:
        def decorate(cls: type[T]) -> type[T]:
            if name in self._entries:
                raise ValueError(f"{self._kind} '{name}' is already registered")
            if not (isinstance(cls, type) and issubclass(cls, self._base)):
                raise TypeError(f"{getattr(cls, '__name__', cls)} must subclass {self._base.__name__}")
            self._entries[name] = cls
            return cls

        return decorate

    def get(self, name: str) -> type[T]:
        if name not in self._entries:
            raise KeyError(f"unknown {self._kind} '{name}'; available: {self.available()}")
        return self._entries[name]

    def build(self, name: str, *args: Any, **kwargs: Any) -> T:
        return self.get(name)(*args, **kwargs)

    def available(self) -> list[str]:
        return sorted(self._entries)

    def __contains__(self, name: object) -> bool:
        return name in self._entries
