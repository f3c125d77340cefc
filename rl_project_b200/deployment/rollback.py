"""Rollback and kill switch (``src/forgeline/deployment/rollback.py:14-51`` behaviour):
retire the champion and restore its rollback target in one step, refusing when
that would leave no champion; or stop routing to one candidate."""

from __future__ import annotations

from typing import Optional

from rl_project_b200.core.errors import RegistryError
from rl_project_b200.deployment.candidates import ALLOWED_TRANSITIONS, CandidateState, ModelCandidate
from rl_project_b200.deployment.registry import CandidateRegistry
from rl_project_b200.deployment.rollout import RoutingPolicy
from rl_project_b200.observability.events import Event


def rollback(registry: CandidateRegistry, name: str, reason: str = "manual rollback",
             routing: Optional[RoutingPolicy] = None) -> ModelCandidate:
    current = registry.champion(name)
    if current is None:
        raise RegistryError(f"no champion to roll back for {name!r}")
    if not current.rollback_target:
        raise RegistryError(f"champion {current.key} has no rollback target")
    target = registry.get(current.rollback_target)
    if CandidateState.CHAMPION not in ALLOWED_TRANSITIONS[target.state]:
        raise RegistryError(f"rollback target {target.key} cannot return from {target.state.value}")
    current.transition(CandidateState.RETIRED, reason=reason)
    target.transition(CandidateState.CHAMPION, reason=f"rollback from {current.id}: {reason}")
    target.rollback_target = None
    registry.update(current)
    registry.update(target)
    if routing is not None:
        routing.champion = target.key
        if routing.challenger in (current.key, target.key):
            routing.challenger, routing.challenger_percent = None, 0.0
        routing.disable_backend(current.key)
    if registry.metrics is not None:
        registry.metrics.event(Event.CANDIDATE_ROLLED_BACK.value, {"from": current.id, "to": target.id,
                                                                   "reason": reason})
    return target


def disable_candidate(registry: CandidateRegistry, candidate_id: str, routing: Optional[RoutingPolicy] = None,
                      reason: str = "disabled") -> ModelCandidate:
    """Kill switch: stop routing to a candidate; its registry state is unchanged."""
    c = registry.get(candidate_id)
    if routing is not None:
        routing.disable_backend(c.key)
    c.tags = sorted(set(c.tags) | {"disabled"})
    c.note(c.state, reason)
    registry.update(c)
    return c
