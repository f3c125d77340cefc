"""Champion / challenger / shadow traffic routing by request-id hash, traffic
simulation and offline replay (behaviour of ``src/forgeline/deployment/rollout.py:14-125``).

``RoutingPolicy.route`` is a valid ``Router`` ``route_fn`` once wrapped with
``as_route_fn`` (it returns the serving backend's name)."""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Sequence, Set

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.deployment.feature_flags import in_percentage, stable_bucket

DEFAULT_SALT = "forgeline-routing"


@dataclass
class RoutingDecision:
    primary: str
    shadow: Optional[str] = None
    bucket: int = 0
    reason: str = ""


@dataclass
class RoutingPolicy:
    """``challenger`` serves ``challenger_percent`` % of requests, ``champion`` the rest;
    ``shadow`` receives a copy of ``shadow_percent`` % (its answer is discarded);
    ``pinned`` maps request ids to a backend; ``disabled`` backends get no traffic."""

    champion: str
    challenger: Optional[str] = None
    challenger_percent: float = 0.0
    shadow: Optional[str] = None
    shadow_percent: float = 0.0
    salt: str = DEFAULT_SALT
    pinned: Dict[str, str] = field(default_factory=dict)
    disabled: Set[str] = field(default_factory=set)

    def validate(self) -> None:
        for pct in (self.challenger_percent, self.shadow_percent):
            if not 0.0 <= pct <= 100.0:
                raise ConfigError("percentages must be in [0, 100]")
        if self.challenger_percent > 0 and not self.challenger:
            raise ConfigError("challenger_percent > 0 requires a challenger backend")
        if self.shadow_percent > 0 and not self.shadow:
            raise ConfigError("shadow_percent > 0 requires a shadow backend")

    def _live(self, name: Optional[str]) -> bool:
        return bool(name) and name not in self.disabled

    def route(self, request_id: str, requested: Optional[str] = None) -> RoutingDecision:
        """First rule that decides wins: an explicitly requested pinned backend, a pin of this request id, then
        the hash split between challenger and champion; the shadow copy is decided independently."""
        self.validate()
        for rule in (self._explicit, self._pinned):
            decision = rule(request_id, requested)
            if decision is not None:
                return decision
        bucket = stable_bucket(request_id, self.salt)
        to_challenger = self._live(self.challenger) and bucket < self.challenger_percent * 100
        primary = self.challenger if to_challenger else self.champion
        reason = f"challenger ({self.challenger_percent}%)" if to_challenger else "champion"
        return RoutingDecision(primary=primary, shadow=self._shadow_for(request_id, primary), bucket=bucket,  # type: ignore[arg-type]
                               reason=reason)

    def _explicit(self, request_id: str, requested: Optional[str]) -> Optional[RoutingDecision]:
        if requested and requested in self.pinned.values() and self._live(requested):
            return RoutingDecision(primary=requested, bucket=-1, reason="explicit model request")
        return None

    def _pinned(self, request_id: str, requested: Optional[str]) -> Optional[RoutingDecision]:
        pin = self.pinned.get(request_id)
        return RoutingDecision(primary=pin, bucket=-1, reason="pinned") if self._live(pin) else None  # type: ignore[arg-type]

    def _shadow_for(self, request_id: str, primary: Optional[str]) -> Optional[str]:
        if self._live(self.shadow) and self.shadow != primary and \
                in_percentage(request_id, self.salt + ":shadow", self.shadow_percent):
            return self.shadow
        return None

    def as_route_fn(self) -> Callable[[str, Optional[str]], str]:
        return lambda request_id, requested: self.route(request_id, requested).primary

    def disable_backend(self, name: str) -> None:
        self.disabled.add(name)

    def enable_backend(self, name: str) -> None:
        self.disabled.discard(name)

    def to_dict(self) -> Dict[str, Any]:
        return {"champion": self.champion, "challenger": self.challenger,
                "challenger_percent": self.challenger_percent, "shadow": self.shadow,
                "shadow_percent": self.shadow_percent, "salt": self.salt, "pinned": dict(self.pinned),
                "disabled": sorted(self.disabled)}

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "RoutingPolicy":
        p = cls(champion=d["champion"], challenger=d.get("challenger"),
                challenger_percent=float(d.get("challenger_percent", 0.0)), shadow=d.get("shadow"),
                shadow_percent=float(d.get("shadow_percent", 0.0)), salt=d.get("salt", DEFAULT_SALT),
                pinned=dict(d.get("pinned", {})), disabled=set(d.get("disabled", [])))
        p.validate()
        return p

    def save(self, path) -> None:
        Path(path).write_text(json.dumps(self.to_dict(), indent=2))

    @classmethod
    def load(cls, path) -> "RoutingPolicy":
        return cls.from_dict(json.loads(Path(path).read_text()))


def simulate_traffic(policy: RoutingPolicy, request_ids: Sequence[str]) -> Dict[str, float]:
    """Fraction of requests each backend would serve, plus the shadowed fraction."""
    counts: Dict[str, int] = {}
    shadowed = 0
    for rid in request_ids:
        d = policy.route(rid)
        counts[d.primary] = counts.get(d.primary, 0) + 1
        shadowed += d.shadow is not None
    n = max(len(request_ids), 1)
    out = {k: v / n for k, v in counts.items()}
    out["shadow_fraction"] = shadowed / n
    return out


@dataclass
class ReplayResult:
    n: int
    per_backend: Dict[str, Dict[str, float]]


def offline_replay(backends: Dict[str, Any], prompts: Sequence[str], scorer, params=None) -> ReplayResult:
    """Send the same prompts to every backend and score each output (offline A/B)."""
    from rl_project_b200.inference.requests import SamplingParams

    params = params or SamplingParams(max_tokens=32, temperature=0.0)
    per: Dict[str, Dict[str, float]] = {}
    for name, backend in backends.items():
        scores: List[float] = [float(scorer(p, backend.complete(p, params, request_id=f"replay-{i}").text))
                               for i, p in enumerate(prompts)]
        per[name] = {"mean_score": sum(scores) / max(len(scores), 1), "n": float(len(scores))}
    return ReplayResult(n=len(prompts), per_backend=per)
