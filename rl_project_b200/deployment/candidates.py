"""Model candidates and their lifecycle state machine.

States and allowed moves follow ``src/forgeline/deployment/candidates.py:14-74``:
experimental -> shadow / challenger -> champion -> retired, with a retired
candidate returning only through an explicit restore (rollback).
"""

from __future__ import annotations

import time
import uuid
from dataclasses import asdict, dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional, Set

from rl_project_b200.core.errors import RegistryError


class CandidateState(str, Enum):
    EXPERIMENTAL = "experimental"
    SHADOW = "shadow"
    CHALLENGER = "challenger"
    CHAMPION = "champion"
    RETIRED = "retired"


_S = CandidateState
ALLOWED_TRANSITIONS: Dict[CandidateState, Set[CandidateState]] = {
    _S.EXPERIMENTAL: {_S.SHADOW, _S.CHALLENGER, _S.RETIRED},
    _S.SHADOW: {_S.CHALLENGER, _S.EXPERIMENTAL, _S.RETIRED},
    _S.CHALLENGER: {_S.CHAMPION, _S.SHADOW, _S.EXPERIMENTAL, _S.RETIRED},
    _S.CHAMPION: {_S.RETIRED, _S.CHALLENGER},
    _S.RETIRED: {_S.CHALLENGER, _S.CHAMPION},  # restore paths only
}


@dataclass
class ModelCandidate:
    name: str
    version: str
    algorithm: str
    checkpoint: str
    tokenizer: str = ""
    dataset: str = ""
    precision: str = "float32"
    distributed_strategy: str = "single"
    model_spec: Dict[str, Any] = field(default_factory=dict)
    metrics: Dict[str, float] = field(default_factory=dict)
    state: CandidateState = CandidateState.EXPERIMENTAL
    id: str = field(default_factory=lambda: uuid.uuid4().hex[:12])
    created_at: float = field(default_factory=time.time)
    updated_at: float = field(default_factory=time.time)
    promotion_status: str = "none"  # none | passed | rejected
    promotion_report: Dict[str, Any] = field(default_factory=dict)
    rollback_target: Optional[str] = None  # id of the candidate to restore on rollback
    tags: List[str] = field(default_factory=list)
    history: List[Dict[str, Any]] = field(default_factory=list)

    @property
    def key(self) -> str:
        return f"{self.name}:{self.version}"

    def note(self, new_state: CandidateState, reason: str) -> None:
        self.history.append({"from": self.state.value, "to": new_state.value, "reason": reason, "ts": time.time()})
        self.updated_at = time.time()

    def transition(self, new_state: CandidateState, reason: str = "") -> None:
        if new_state not in ALLOWED_TRANSITIONS[self.state]:
            raise RegistryError(f"cannot move candidate {self.key} from {self.state.value} to {new_state.value}")
        self.note(new_state, reason)
        self.state = new_state

    def to_dict(self) -> Dict[str, Any]:
        d = asdict(self)
        d["state"] = self.state.value
        return d

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "ModelCandidate":
        d = dict(d)
        d["state"] = CandidateState(d.get("state", "experimental"))
        return cls(**d)
