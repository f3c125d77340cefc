"""Deployment life cycle: registry, promotion gates, flags, routing, rollback."""
from __future__ import annotations

import json

import pytest

from rl_project_b200.core.errors import ConfigError, PromotionError, RegistryError
from rl_project_b200.deployment import (CandidateRegistry, CandidateState, FeatureFlag, FeatureFlags, GateRule,
                                        ModelCandidate, PromotionGate, RoutingPolicy, disable_candidate,
                                        offline_replay, rollback, simulate_traffic, stable_bucket)


def _cand(version, **kw):
    return ModelCandidate(name="m", version=version, algorithm="sft", checkpoint=f"/ckpt/{version}", **kw)


def test_state_machine_and_registry_persistence(tmp_path):
    path = tmp_path / "reg.json"
    reg = CandidateRegistry(path)
    a = reg.register(_cand("1"))
    with pytest.raises(RegistryError):
        reg.register(_cand("1"))
    with pytest.raises(RegistryError):
        reg.transition(a.id, CandidateState.CHAMPION)  # experimental -> champion is not allowed
    reg.transition(a.id, CandidateState.CHALLENGER)
    reg.transition(a.id, CandidateState.CHAMPION)
    b = reg.register(_cand("2"))
    reg.transition(b.id, CandidateState.CHALLENGER)
    reg.transition(b.id, CandidateState.CHAMPION)
    assert reg.champion("m").id == b.id and reg.get(a.id).state == CandidateState.RETIRED
    assert reg.get(b.id).rollback_target == a.id
    reloaded = CandidateRegistry(path)
    assert reloaded.champion("m").id == b.id and len(reloaded.list()) == 2
    assert json.loads(path.read_text())["format_version"] == 1
    reg.record_metrics(b.id, {"acc": 0.9})
    assert CandidateRegistry(path).get(b.id).metrics["acc"] == 0.9
    path.write_text("{broken")
    with pytest.raises(RegistryError):
        CandidateRegistry(path)


def test_rollback_and_kill_switch(tmp_path):
    reg = CandidateRegistry(tmp_path / "r.json")
    a, b = reg.register(_cand("1")), reg.register(_cand("2"))
    for c in (a, b):
        reg.transition(c.id, CandidateState.CHALLENGER)
        reg.transition(c.id, CandidateState.CHAMPION)
    routing = RoutingPolicy(champion=b.key, challenger=a.key, challenger_percent=10)
    restored = rollback(reg, "m", routing=routing)
    assert restored.id == a.id and reg.champion("m").id == a.id
    assert routing.champion == a.key and routing.challenger is None and b.key in routing.disabled
    with pytest.raises(RegistryError):
        rollback(reg, "m")  # the restored champion has no rollback target
    c = disable_candidate(reg, a.id, routing)
    assert "disabled" in c.tags and a.key in routing.disabled and c.state == CandidateState.CHAMPION


def test_promotion_gate_fails_closed():
    gate = PromotionGate([GateRule("acc", min=0.5), GateRule("acc", min_delta=0.01),
                          GateRule("latency", max_increase=0.1, relative=True)])
    assert gate.evaluate({"acc": 0.7, "latency": 1.05}, {"acc": 0.65, "latency": 1.0}).passed
    rep = gate.evaluate({"acc": 0.66, "latency": 1.2}, {"acc": 0.65, "latency": 1.0})
    assert not rep.passed and {c.metric for c in rep.failures()} == {"latency"}
    assert not gate.evaluate({"acc": float("nan"), "latency": 1.0}, {"acc": 0.1, "latency": 1.0}).passed
    assert not gate.evaluate({"acc": 0.9, "latency": 1.0}).passed  # relative rules need an incumbent
    lenient = PromotionGate(gate.rules, when_no_baseline="skip_relative")
    assert lenient.evaluate({"acc": 0.9, "latency": 1.0}).passed
    assert not lenient.evaluate({"acc": 0.4, "latency": 1.0}).passed  # absolute rules still apply
    with pytest.raises(PromotionError):
        gate.assert_promotable({"acc": 0.1})
    with pytest.raises(ConfigError):
        PromotionGate.from_config({"rules": [{"metric": "x"}]})
    with pytest.raises(ConfigError):
        PromotionGate.from_config({"rules": []})
    strict = PromotionGate.from_config({"rules": [{"metric": "x", "min": 0}], "require_baseline": True})
    assert not strict.evaluate({"x": 1.0}).passed


def test_feature_flags(tmp_path):
    assert stable_bucket("user-1", "s") == stable_bucket("user-1", "s")
    flags = FeatureFlags(tmp_path / "flags.json")
    flags.set(FeatureFlag("new_sampler", percentage=30.0, allow={"vip"}, deny={"bad"}))
    on = sum(flags.is_on("new_sampler", f"u{i}") for i in range(4000)) / 4000
    assert 0.25 < on < 0.35
    assert flags.is_on("new_sampler", "vip") and not flags.is_on("new_sampler", "bad")
    assert not flags.is_on("new_sampler") and flags.is_on("missing", default=True)
    flags.disable("new_sampler")
    assert not FeatureFlags(tmp_path / "flags.json").is_on("new_sampler", "vip")
    with pytest.raises(ConfigError):
        FeatureFlag("x", percentage=120).validate()


def test_routing_policy_and_replay():
    from rl_project_b200.serving import EchoBackend, Router

    p = RoutingPolicy(champion="a", challenger="b", challenger_percent=20, shadow="c", shadow_percent=50,
                      pinned={"req-pin": "c"})
    frac = simulate_traffic(p, [f"r{i}" for i in range(5000)])
    assert 0.17 < frac["b"] < 0.23 and 0.45 < frac["shadow_fraction"] < 0.55
    assert p.route("req-pin").primary == "c" and p.route("x", requested="c").reason == "explicit model request"
    p.disable_backend("b")
    assert simulate_traffic(p, [f"r{i}" for i in range(500)]).get("b", 0) == 0
    back = RoutingPolicy.from_dict(p.to_dict())
    assert back.to_dict() == p.to_dict()
    with pytest.raises(ConfigError):
        RoutingPolicy(champion="a", challenger_percent=5).validate()
    router = Router({"a": EchoBackend("a"), "b": EchoBackend("b"), "c": EchoBackend("c")}, "a",
                    route_fn=p.as_route_fn())
    st, out = router.handle("POST", "/v1/completions", {"prompt": "hi", "request_id": "req-pin"})
    assert st == 200 and out["forgeline"]["backend"] == "c"
    rep = offline_replay({"a": EchoBackend("a")}, ["abc", "de"], lambda p, o: float(o == p[::-1]))
    assert rep.per_backend["a"]["mean_score"] == 1.0 and rep.n == 2
