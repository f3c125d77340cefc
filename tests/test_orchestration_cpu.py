"""Worker pools on the in-process thread backend: sharding, order, recovery, weight sync."""
from __future__ import annotations

import importlib.util

import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.core.errors import OptionalDependencyError, OrchestrationError
from rl_project_b200.core.protocols import RewardResult, Trajectory
from rl_project_b200.data.tokenizers import CharTokenizer
from rl_project_b200.models.policy import NativePolicy
from rl_project_b200.models.transformer.model import TransformerLM
from rl_project_b200.orchestration.config import RayConfig
from rl_project_b200.orchestration.pools import (EvaluatorPool, RewardPool, RolloutPool, ThreadBackend, ToolPool,
                                                 WorkerPool, chunks, weights_version)
from rl_project_b200.rollouts.engine import RolloutConfig

CFG = RayConfig(backend="threads", max_call_retries=2)


class LenReward:
    def score(self, t: Trajectory) -> RewardResult:
        return RewardResult(value=float(len(t.response_text)))


class Boom:
    def score(self, t):
        raise ValueError("user code failed")


def _traj(text: str) -> Trajectory:
    return Trajectory(prompt_ids=torch.tensor([1]), response_ids=torch.tensor([2]), response_text=text)


def test_chunks():
    assert chunks(list(range(7)), 3) == [[0, 1, 2], [3, 4], [5, 6]]
    assert chunks([1], 4) == [[1]]


def test_reward_pool_order_and_recovery():
    pool = RewardPool(LenReward(), 3, CFG)
    trajs = [_traj("x" * i) for i in range(10)]
    assert [r.value for r in pool.score_many(trajs)] == [float(i) for i in range(10)]
    ThreadBackend.crash(pool.workers[1])  # the next call to worker 1 finds it dead
    assert [r.value for r in pool.score_many(trajs)] == [float(i) for i in range(10)]
    assert pool.restarts == 1 and pool.generations == [0, 1, 0]
    bad = RewardPool(Boom(), 2, CFG)
    with pytest.raises(ValueError):  # user errors are not retried
        bad.score_many(trajs)
    assert bad.restarts == 0
    pool.shutdown()


def test_retries_are_bounded():
    class Dying(WorkerPool):
        def _spawn(self, index):
            h = super()._spawn(index)
            ThreadBackend.crash(h)  # every replacement is dead on arrival
            return h

    pool = Dying(1, RayConfig(backend="threads", max_call_retries=2))
    pool.workers, pool.generations = [pool._spawn(0)], [0]
    with pytest.raises(OrchestrationError):
        pool.broadcast("ping")
    assert pool.restarts == 2


def test_tool_pool():
    pool = ToolPool(2, CFG, timeout=10.0)
    out = pool.execute_many(["print(1+1)", "raise SystemExit(3)", "print('ok')"])
    assert out[0]["output"].strip() == "2" and out[2]["output"].strip() == "ok" and out[1]["error"]


@pytest.fixture
def policy():
    torch.manual_seed(0)
    tok = CharTokenizer.ascii()
    return NativePolicy(TransformerLM(model_spec_from_preset("tiny", vocab_size=tok.vocab_size)), tok)


def test_rollout_pool_weight_sync(policy):
    cfg = RolloutConfig(group_size=3, max_new_tokens=4, temperature=0.0, engine="generate", record_old_logprobs=False)
    pool = RolloutPool(policy, cfg, 2, CFG)
    v0 = weights_version(policy.model)
    assert pool.worker_versions() == [v0, v0] and pool.weight_pushes == 1
    group = pool.rollout(torch.tensor([5, 6, 7]))
    assert len(group) == 3 and len({tuple(t.response_ids.tolist()) for t in group}) == 1  # greedy
    assert not pool.sync_weights()  # unchanged parameters: nothing pushed
    with torch.no_grad():
        for p in policy.model.parameters():
            p.add_(0.01)
    many = pool.rollout_many([torch.tensor([1, 2]), torch.tensor([3, 4])])
    assert pool.weight_pushes == 2 and pool.worker_versions() == [weights_version(policy.model)] * 2
    assert [len(g) for g in many] == [3, 3]
    ThreadBackend.crash(pool.workers[0])
    pool.rollout(torch.tensor([5, 6, 7]))
    assert pool.restarts == 1 and pool.worker_versions()[0] == weights_version(policy.model)  # restored weights


def test_evaluator_pool_matches_single_process(tmp_path, policy):
    from rl_project_b200.checkpoints.manager import CheckpointManager, CheckpointState
    from rl_project_b200.evaluation.suites import BenchmarkSuite, build_benchmark

    mgr = CheckpointManager(tmp_path / "ck")
    path = mgr.save(CheckpointState(model_state=policy.model.state_dict(), step=1, algorithm="sft",
                                    model_spec=policy.model.spec.to_dict(), tokenizer_meta=policy.tokenizer.metadata()))
    ev = EvaluatorPool(str(path), 2, CFG)
    merged = ev.run("arc", max_new_tokens=3)
    single = BenchmarkSuite(build_benchmark("arc"), max_new_tokens=3).run(ev.workers[0].obj.policy)
    assert [i["index"] for i in merged.per_item] == [0, 1, 2]
    assert merged.metrics["accuracy"] == single.metrics["accuracy"] and merged.details["workers"] == 2


def test_attach_through_manifest():
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.training.factory import build_algorithm

    m = ExperimentManifest.from_dict({
        "name": "orch", "algorithm": "grpo", "model_preset": "tiny", "model": {"vocab_size": 256, "block_size": 64},
        "data": {"kind": "verifiable", "path": "synthetic:addition", "tokenizer": "byte", "extra": {"n_tasks": 8}},
        "reward": {"type": "verifier", "verifier": "math"},
        "algorithm_params": {"group_size": 2, "prompts_per_step": 2,
                             "rollout": {"max_new_tokens": 4, "engine": "generate"}},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": 1, "batch_size": 2},
        "orchestration": {"type": "ray", "backend": "threads", "reward_workers": 2, "rollout_workers": 2},
        "output_dir": "/tmp/rlb_orch_test"})
    ctx = RunContext.create(m, metrics_backend="none")
    alg = build_algorithm(m, ctx)
    assert type(alg.reward).__name__ == "RewardPool" and type(alg.rollouts).__name__ == "RolloutPool"
    batch = alg.collect(0)
    loss, _ = alg.loss(batch, 0, 1)
    assert torch.isfinite(loss)


@pytest.mark.skipif(importlib.util.find_spec("ray") is not None, reason="Ray is installed")
def test_ray_backend_reports_missing_dependency():
    with pytest.raises(OptionalDependencyError):
        import rl_project_b200.orchestration.ray_backend  # noqa: F401
