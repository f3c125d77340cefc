"""Local JSON-backed candidate registry with atomic writes and a single champion per name.

File format ``{"format_version": 1, "candidates": [...]}`` as in
``src/forgeline/deployment/registry.py:19-101`` so registries move between the
two frameworks.  Writes are serialised by a lock and land atomically.
"""

from __future__ import annotations

import json
import os
import threading
from pathlib import Path
from typing import Dict, List, Optional

from rl_project_b200.core.errors import RegistryError
from rl_project_b200.deployment._io import write_json_atomic
from rl_project_b200.deployment.candidates import CandidateState, ModelCandidate
from rl_project_b200.observability.events import Event
from rl_project_b200.observability.logging import get_logger

log = get_logger("forgeline.registry")


class CandidateRegistry:
    def __init__(self, path: str | os.PathLike, metrics=None):
        self.path = Path(path)
        self.metrics = metrics
        self._candidates: Dict[str, ModelCandidate] = {}
        self._lock = threading.RLock()
        if self.path.exists():
            self._load()

    def _load(self) -> None:
        try:
            data = json.loads(self.path.read_text())
        except json.JSONDecodeError as exc:
            raise RegistryError(f"registry file {self.path} is corrupt: {exc}") from None
        self._candidates = {c["id"]: ModelCandidate.from_dict(c) for c in data.get("candidates", [])}

    def _save(self) -> None:
        write_json_atomic(self.path, {"format_version": 1,
                                      "candidates": [c.to_dict() for c in self._candidates.values()]})

    def _event(self, name: str, payload: dict) -> None:
        if self.metrics is not None:
            self.metrics.event(name, payload)

    def register(self, candidate: ModelCandidate) -> ModelCandidate:
        with self._lock:
            if any(c.key == candidate.key for c in self._candidates.values()):
                raise RegistryError(f"candidate {candidate.key} already registered")
            self._candidates[candidate.id] = candidate
            self._save()
        self._event(Event.CANDIDATE_REGISTERED.value, {"id": candidate.id, "key": candidate.key})
        log.info("candidate_registered", id=candidate.id, key=candidate.key)
        return candidate

    def get(self, candidate_id: str) -> ModelCandidate:
        c = self._candidates.get(candidate_id)
        if c is None:
            raise RegistryError(f"unknown candidate id {candidate_id!r}")
        return c

    def find(self, name: str, version: Optional[str] = None) -> List[ModelCandidate]:
        return [c for c in self._candidates.values() if c.name == name and version in (None, c.version)]

    def list(self, state: Optional[CandidateState] = None, name: Optional[str] = None) -> List[ModelCandidate]:
        out = [c for c in self._candidates.values() if state in (None, c.state) and name in (None, c.name)]
        return sorted(out, key=lambda c: c.created_at)

    def update(self, candidate: ModelCandidate) -> None:
        with self._lock:
            if candidate.id not in self._candidates:
                raise RegistryError(f"unknown candidate id {candidate.id!r}")
            self._candidates[candidate.id] = candidate
            self._save()

    def record_metrics(self, candidate_id: str, metrics: Dict[str, float]) -> ModelCandidate:
        with self._lock:
            c = self.get(candidate_id)
            c.metrics.update({k: float(v) for k, v in metrics.items()})
            self.update(c)
        return c

    def champion(self, name: str) -> Optional[ModelCandidate]:
        champs = [c for c in self._candidates.values() if c.name == name and c.state == CandidateState.CHAMPION]
        if len(champs) > 1:
            raise RegistryError(f"registry has {len(champs)} champions for {name!r}; expected at most one")
        return champs[0] if champs else None

    def transition(self, candidate_id: str, new_state: CandidateState, reason: str = "") -> ModelCandidate:
        """Move a candidate; promoting a champion retires the incumbent and records it as rollback target."""
        with self._lock:
            c = self.get(candidate_id)
            if new_state == CandidateState.CHAMPION:
                incumbent = self.champion(c.name)
                if incumbent is not None and incumbent.id != c.id:
                    c.transition(new_state, reason)  # validate before touching the incumbent
                    incumbent.transition(CandidateState.RETIRED, reason=f"replaced by {c.id}")
                    c.rollback_target = incumbent.id
                    self._save()
                    self._event(Event.CANDIDATE_PROMOTED.value, {"id": c.id, "replaced": incumbent.id})
                    return c
            c.transition(new_state, reason)
            self._save()
        if new_state == CandidateState.CHAMPION:
            self._event(Event.CANDIDATE_PROMOTED.value, {"id": c.id})
        return c

    def retire(self, candidate_id: str, reason: str = "") -> ModelCandidate:
        return self.transition(candidate_id, CandidateState.RETIRED, reason)
