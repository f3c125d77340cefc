"""Rollback and kill switch (behaviour of ``src/forgeline/deployment/rollback.py``).

``rollback`` retires a model's champion and restores its recorded rollback target as champion in ONE
registry commit (both candidates change together or neither does); it refuses when there is no champion,
no target, or the target's state cannot return to champion.  ``disable_candidate`` stops routing to one
candidate and tags it, leaving its lifecycle state alone.
"""

from __future__ import annotations

from typing import Optional

from rl_project_b200.core.errors import RegistryError
from rl_project_b200.deployment.candidates import CandidateState, ModelCandidate, can_move
from rl_project_b200.deployment.registry import CandidateRegistry
from rl_project_b200.deployment.rollout import RoutingPolicy
from rl_project_b200.observability.events import Event


def _reroute(routing: RoutingPolicy, retired_key: str, restored_key: str) -> None:
    routing.champion = restored_key
    if routing.challenger in (retired_key, restored_key):
        routing.challenger, routing.challenger_percent = None, 0.0
    routing.disable_backend(retired_key)


def rollback(registry: CandidateRegistry, name: str, reason: str = "manual rollback",
             routing: Optional[RoutingPolicy] = None) -> ModelCandidate:
    current = registry.champion(name)
    if current is None:
        raise RegistryError(f"no champion to roll back for {name!r}")
    if not current.rollback_target:
        raise RegistryError(f"champion {current.key} has no rollback target")
    retired_id, target_id = current.id, current.rollback_target

    def swap(table):
        old, target = table[retired_id], registry._lookup(table, target_id)
        if not can_move(target.state, CandidateState.CHAMPION):
            raise RegistryError(f"rollback target {target.key} cannot return from {target.state.value}")
        old.transition(CandidateState.RETIRED, reason=reason)
        target.transition(CandidateState.CHAMPION, reason=f"rollback from {retired_id}: {reason}")
        target.rollback_target = None
        return target

    restored = registry._commit(swap)
    if routing is not None:
        _reroute(routing, current.key, restored.key)
    registry._event(Event.CANDIDATE_ROLLED_BACK.value, {"from": retired_id, "to": restored.id, "reason": reason})
    return restored


def disable_candidate(registry: CandidateRegistry, candidate_id: str, routing: Optional[RoutingPolicy] = None,
                      reason: str = "disabled") -> ModelCandidate:
    """Kill switch: no more traffic to the candidate; its registry state is unchanged."""
    def tag(table):
        c = registry._lookup(table, candidate_id)
        c.tags = sorted({*c.tags, "disabled"})
        c.note(c.state, reason)
        return c

    c = registry._commit(tag)
    if routing is not None:
        routing.disable_backend(c.key)
    return c
