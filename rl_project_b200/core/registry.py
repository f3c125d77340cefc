"""Named registries of factories (the contract of ``src/forgeline/core/registry.py:12-50``).

A ``Registry`` maps names to objects of one kind (algorithms, verifiers, reward providers, ...).  ``register``
works as a call (``reg.register("x", obj)``) or a decorator (``@reg.register("x")``); registering a name twice
and looking up an unknown name are configuration errors that list what is registered.  Iteration yields the
names in sorted order.
"""

from __future__ import annotations

from typing import Callable, Dict, Generic, Iterator, Optional, TypeVar

from rl_project_b200.core.errors import ConfigError

T = TypeVar("T")


class Registry(Generic[T]):
    def __init__(self, kind: str):
        self.kind = kind
        self._table: Dict[str, T] = {}

    def _insert(self, name: str, obj: T) -> T:
        if name in self._table:
            raise ConfigError(f"{self.kind} {name!r} is already registered")
        self._table[name] = obj
        return obj

    def register(self, name: str, item: Optional[T] = None):
        if item is not None:
            return self._insert(name, item)
        return lambda obj: self._insert(name, obj)

    def get(self, name: str) -> T:
        found = self._table.get(name)
        if found is None and name not in self._table:
            raise ConfigError(f"Unknown {self.kind} {name!r}. Registered: {self.names()}")
        return found  # type: ignore[return-value]

    def names(self) -> list[str]:
        return sorted(self._table)

    def __contains__(self, name: object) -> bool:
        return name in self._table

    def __iter__(self) -> Iterator[str]:
        return iter(self.names())

    def __len__(self) -> int:
        return len(self._table)


Factory = Callable[..., T]
