"""Local JSON-backed registry of model candidates, with at most one champion per model name.

The file is ``{"format_version": 1, "candidates": [...]}`` (the format of
``src/forgeline/deployment/registry.py``, so registries move between the two frameworks).

Every change goes through ``_commit``: under the registry lock it applies a mutation to an in-memory copy
of the candidate table, validates the one-champion invariant on the result, writes the file atomically and
only then swaps the copy in -- a failed transition or write leaves both the file and the in-memory state
as they were.  Events are emitted after the commit.
"""

from __future__ import annotations

import copy
import json
import os
import threading
from pathlib import Path
from typing import Callable, Dict, List, Optional

from rl_project_b200.core.errors import RegistryError
from rl_project_b200.deployment._io import write_json_atomic
from rl_project_b200.deployment.candidates import CandidateState, ModelCandidate
from rl_project_b200.observability.events import Event
from rl_project_b200.observability.logging import get_logger

log = get_logger("forgeline.registry")

Table = Dict[str, ModelCandidate]


def _champions(table: Table, name: str) -> List[ModelCandidate]:
    return [c for c in table.values() if c.name == name and c.state == CandidateState.CHAMPION]


class CandidateRegistry:
    def __init__(self, path: str | os.PathLike, metrics=None):
        self.path = Path(path)
        self.metrics = metrics
        self._lock = threading.RLock()
        self._candidates: Table = self._read() if self.path.exists() else {}

    # ------------------------------------------------------------ storage
    def _read(self) -> Table:
        try:
            data = json.loads(self.path.read_text())
        except json.JSONDecodeError as exc:
            raise RegistryError(f"registry file {self.path} is corrupt: {exc}") from None
        return {d["id"]: ModelCandidate.from_dict(d) for d in data.get("candidates", [])}

    def _commit(self, mutate: Callable[[Table], ModelCandidate]) -> ModelCandidate:
        with self._lock:
            draft = copy.deepcopy(self._candidates)
            result = mutate(draft)
            for name in {c.name for c in draft.values()}:
                if len(_champions(draft, name)) > 1:
                    raise RegistryError(f"registry would hold several champions for {name!r}")
            write_json_atomic(self.path, {"format_version": 1, "candidates": [c.to_dict() for c in draft.values()]})
            self._candidates = draft
            return self._candidates[result.id]

    def _event(self, name: str, payload: dict) -> None:
        if self.metrics is not None:
            self.metrics.event(name, payload)

    # ------------------------------------------------------------ queries
    def get(self, candidate_id: str) -> ModelCandidate:
        return self._lookup(self._candidates, candidate_id)

    @staticmethod
    def _lookup(table: Table, candidate_id: str) -> ModelCandidate:
        if candidate_id not in table:
            raise RegistryError(f"unknown candidate id {candidate_id!r}")
        return table[candidate_id]

    def find(self, name: str, version: Optional[str] = None) -> List[ModelCandidate]:
        return [c for c in self._candidates.values() if c.name == name and version in (None, c.version)]

    def list(self, state: Optional[CandidateState] = None, name: Optional[str] = None) -> List[ModelCandidate]:
        keep = [c for c in self._candidates.values() if state in (None, c.state) and name in (None, c.name)]
        return sorted(keep, key=lambda c: c.created_at)

    def champion(self, name: str) -> Optional[ModelCandidate]:
        champs = _champions(self._candidates, name)
        if len(champs) > 1:
            raise RegistryError(f"registry has {len(champs)} champions for {name!r}; expected at most one")
        return champs[0] if champs else None

    # ------------------------------------------------------------ changes
    def register(self, candidate: ModelCandidate) -> ModelCandidate:
        def add(t: Table) -> ModelCandidate:
            if any(c.key == candidate.key for c in t.values()):
                raise RegistryError(f"candidate {candidate.key} already registered")
            t[candidate.id] = candidate
            return candidate

        out = self._commit(add)
        self._event(Event.CANDIDATE_REGISTERED.value, {"id": out.id, "key": out.key})
        log.info("candidate_registered", id=out.id, key=out.key)
        return out

    def update(self, candidate: ModelCandidate) -> None:
        def replace(t: Table) -> ModelCandidate:
            self._lookup(t, candidate.id)
            t[candidate.id] = copy.deepcopy(candidate)
            return candidate

        self._commit(replace)

    def record_metrics(self, candidate_id: str, metrics: Dict[str, float]) -> ModelCandidate:
        def merge(t: Table) -> ModelCandidate:
            c = self._lookup(t, candidate_id)
            c.metrics.update({k: float(v) for k, v in metrics.items()})
            return c

        return self._commit(merge)

    def transition(self, candidate_id: str, new_state: CandidateState, reason: str = "") -> ModelCandidate:
        """Move a candidate.  Promotion to champion retires the incumbent of the same name and records it as
        the new champion's rollback target."""
        replaced: List[str] = []

        def move(t: Table) -> ModelCandidate:
            c = self._lookup(t, candidate_id)
            c.transition(new_state, reason)  # validates the move first
            if new_state == CandidateState.CHAMPION:
                for old in _champions(t, c.name):
                    if old.id != c.id:
                        old.transition(CandidateState.RETIRED, reason=f"replaced by {c.id}")
                        c.rollback_target = old.id
                        replaced.append(old.id)
            return c

        out = self._commit(move)
        if new_state == CandidateState.CHAMPION:
            self._event(Event.CANDIDATE_PROMOTED.value, {"id": out.id, **({"replaced": replaced[0]} if replaced else {})})
        return out

    def retire(self, candidate_id: str, reason: str = "") -> ModelCandidate:
        return self.transition(candidate_id, CandidateState.RETIRED, reason)
