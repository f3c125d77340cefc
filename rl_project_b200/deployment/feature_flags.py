"""Local feature flags with deterministic percentage rollout.

``stable_bucket`` maps ``sha256("salt:key")`` to one of 10,000 buckets, the same
assignment as ``src/forgeline/deployment/feature_flags.py:16-20``, so users keep
their rollout cohort when a deployment moves between the two frameworks.
"""

from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Set

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.deployment._io import write_json_atomic

BUCKETS = 10_000


def stable_bucket(key: str, salt: str = "", buckets: int = BUCKETS) -> int:
    digest = hashlib.sha256(f"{salt}:{key}".encode()).digest()
    return int.from_bytes(digest[:8], "big") % buckets


def in_percentage(key: str, salt: str, percentage: float) -> bool:
    """True for ``percentage`` % of keys (0..100), decided by the key's bucket."""
    return stable_bucket(key, salt) < percentage * (BUCKETS / 100.0)


@dataclass
class FeatureFlag:
    name: str
    enabled: bool = True
    percentage: float = 100.0
    allow: Set[str] = field(default_factory=set)
    deny: Set[str] = field(default_factory=set)
    salt: str = ""
    description: str = ""

    def validate(self) -> None:
        if not 0.0 <= self.percentage <= 100.0:
            raise ConfigError(f"flag {self.name!r}: percentage must be in [0, 100]")

    def is_on(self, key: Optional[str] = None) -> bool:
        """Disabled flags are off; a key on the deny / allow list is off / on; otherwise the percentage
        decides (all, none, or the key's stable bucket -- a flag below 100 % is off for anonymous calls)."""
        if not self.enabled:
            return False
        listed = None if key is None else (False if key in self.deny else (True if key in self.allow else None))
        if listed is not None:
            return listed
        if self.percentage >= 100.0 or self.percentage <= 0.0 or key is None:
            return self.percentage >= 100.0
        return in_percentage(key, self.salt or self.name, self.percentage)

    def to_dict(self) -> Dict[str, Any]:
        return {"name": self.name, "enabled": self.enabled, "percentage": self.percentage,
                "allow": sorted(self.allow), "deny": sorted(self.deny), "salt": self.salt,
                "description": self.description}

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "FeatureFlag":
        f = cls(name=d["name"], enabled=bool(d.get("enabled", True)), percentage=float(d.get("percentage", 100.0)),
                allow=set(d.get("allow", [])), deny=set(d.get("deny", [])), salt=d.get("salt", ""),
                description=d.get("description", ""))
        f.validate()
        return f


class FeatureFlags:
    """Flag set kept in memory, persisted as JSON when a path is given."""

    def __init__(self, path: Optional[str | os.PathLike] = None):
        self.path = Path(path) if path else None
        self._flags: Dict[str, FeatureFlag] = {}
        if self.path and self.path.exists():
            data = json.loads(self.path.read_text())
            self._flags = {f["name"]: FeatureFlag.from_dict(f) for f in data.get("flags", [])}

    def _save(self) -> None:
        if self.path is not None:
            write_json_atomic(self.path, {"flags": [f.to_dict() for f in self._flags.values()]})

    def set(self, flag: FeatureFlag) -> FeatureFlag:
        flag.validate()
        self._flags[flag.name] = flag
        self._save()
        return flag

    def get(self, name: str) -> Optional[FeatureFlag]:
        return self._flags.get(name)

    def is_on(self, name: str, key: Optional[str] = None, default: bool = False) -> bool:
        flag = self._flags.get(name)
        return flag.is_on(key) if flag is not None else default

    def _set_enabled(self, name: str, value: bool) -> None:
        if name in self._flags:
            self._flags[name].enabled = value
            self._save()

    def disable(self, name: str) -> None:
        self._set_enabled(name, False)

    def enable(self, name: str) -> None:
        self._set_enabled(name, True)

    def names(self) -> List[str]:
        return sorted(self._flags)
