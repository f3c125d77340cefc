"""Named factory registry (``src/forgeline/core/registry.py:12-50`` semantics)."""

from __future__ import annotations

from typing import Callable, Dict, Generic, Iterator, Optional, TypeVar

from rl_project_b200.core.errors import ConfigError

T = TypeVar("T")


class Registry(Generic[T]):
    def __init__(self, kind: str):
        self.kind = kind
        self._table: Dict[str, T] = {}

    def register(self, name: str, item: Optional[T] = None):
        def add(obj: T) -> T:
            if name in self._table:
                raise ConfigError(f"{self.kind} {name!r} is already registered")
            self._table[name] = obj
            return obj

        return add(item) if item is not None else add

    def get(self, name: str) -> T:
        if name not in self._table:
            raise ConfigError(f"Unknown {self.kind} {name!r}. Registered: {self.names()}")
        return self._table[name]

    def names(self) -> list[str]:
        return sorted(self._table)

    def __contains__(self, name: object) -> bool:
        return name in self._table

    def __iter__(self) -> Iterator[str]:
        return iter(self.names())

    def __len__(self) -> int:
        return len(self._table)


Factory = Callable[..., T]
