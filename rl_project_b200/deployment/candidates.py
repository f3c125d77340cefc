"""Model candidates and their lifecycle state machine.

States and allowed moves are those of ``src/forgeline/deployment/candidates.py``
(experimental -> shadow / challenger -> champion -> retired, a retired candidate
returning only through an explicit restore), written down as an edge list that
is parsed into the transition table.
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


# the lifecycle graph, one "from -> to, to, ..." line per state (retired returns only by restore / rollback)
_GRAPH = """
experimental -> shadow, challenger, retired
shadow       -> challenger, experimental, retired
challenger   -> champion, shadow, experimental, retired
champion     -> retired, challenger
retired      -> challenger, champion
"""


def _edges(spec: str) -> Dict[CandidateState, Set[CandidateState]]:
    graph: Dict[CandidateState, Set[CandidateState]] = {}
    for line in filter(None, (ln.strip() for ln in spec.splitlines())):
        src, _, dsts = line.partition("->")
        graph[CandidateState(src.strip())] = {CandidateState(d.strip()) for d in dsts.split(",")}
    return graph


ALLOWED_TRANSITIONS: Dict[CandidateState, Set[CandidateState]] = _edges(_GRAPH)


def can_move(src: CandidateState, dst: CandidateState) -> bool:
    return dst in ALLOWED_TRANSITIONS[src]


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
        if not can_move(self.state, new_state):
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
