"""Model life cycle: candidate registry, promotion gates, feature flags, staged rollout, rollback."""

from rl_project_b200.deployment.candidates import ALLOWED_TRANSITIONS, CandidateState, ModelCandidate
from rl_project_b200.deployment.feature_flags import FeatureFlag, FeatureFlags, stable_bucket
from rl_project_b200.deployment.promotion import GateRule, PromotionGate, PromotionReport
from rl_project_b200.deployment.registry import CandidateRegistry
from rl_project_b200.deployment.rollback import disable_candidate, rollback
from rl_project_b200.deployment.rollout import RoutingDecision, RoutingPolicy, offline_replay, simulate_traffic

__all__ = ["ALLOWED_TRANSITIONS", "CandidateState", "ModelCandidate", "FeatureFlag", "FeatureFlags", "stable_bucket",
           "GateRule", "PromotionGate", "PromotionReport", "CandidateRegistry", "disable_candidate", "rollback",
           "RoutingDecision", "RoutingPolicy", "offline_replay", "simulate_traffic"]
