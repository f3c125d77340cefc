"""Quality evaluators: held-out loss / perplexity, verifier pass rate, agent accuracy
(``src/forgeline/evaluation/quality.py:16-89`` metrics).  Every suite works on the whole task list at
once: the pass-rate suite decodes all tasks in one batched rollout and scores them in one batch, the agent
suite runs all episodes in lock-step, and the held-out loss is read back once for all batches."""

from __future__ import annotations

import math
from typing import Any, Dict, List, Optional, Sequence

import torch

from rl_project_b200.core.protocols import EvaluationResult, RewardProvider
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine


class HeldOutLossSuite:
    name = "heldout_loss"

    def __init__(self, corpus, batches: int = 20, batch_size: int = 8, seed: int = 0):
        self.corpus, self.batches, self.batch_size = corpus, batches, batch_size
        self.gen = torch.Generator().manual_seed(seed)

    @torch.no_grad()
    def run(self, model, **kwargs: Any) -> EvaluationResult:
        was = model.training
        model.eval()
        device = next(model.parameters()).device
        total = torch.zeros((), device=device)
        for _ in range(self.batches):
            x, y = self.corpus.sample_batch(self.batch_size, device, self.gen)
            _, loss = model(x, y)
            total += loss.float()
        model.train(was)
        mean = float(total) / self.batches  # one read-back for all batches
        return EvaluationResult(self.name, {"loss": mean, "perplexity": math.exp(min(mean, 50.0))},
                                n_samples=self.batches * self.batch_size)


class VerifierPassRateSuite:
    """Decode every task once (greedy by default), score with a reward provider."""

    name = "verifier_pass_rate"

    def __init__(self, tasks: Sequence[Any], reward: RewardProvider, max_new_tokens: int = 64,
                 temperature: float = 0.0, limit: Optional[int] = None):
        self.tasks = list(tasks)[: limit or None]
        self.reward = reward
        self.config = RolloutConfig(group_size=1, max_new_tokens=max_new_tokens, temperature=temperature,
                                    record_old_logprobs=False)

    @torch.no_grad()
    def run(self, policy, **kwargs: Any) -> EvaluationResult:
        engine = RolloutEngine(policy, self.config)
        prompts = [torch.tensor(policy.encode(t.prompt), dtype=torch.long) for t in self.tasks]
        groups = engine.rollout_many(prompts, tasks=[t.to_dict() for t in self.tasks],
                                     prompt_texts=[t.prompt for t in self.tasks]) if self.tasks else []
        from rl_project_b200.rollouts.rewards.composite import batch_scores

        trajs = [g[0] for g in groups]
        per_item: List[Dict[str, Any]] = []
        passed = malformed = 0
        total = 0.0
        for task, traj, r in zip(self.tasks, trajs, batch_scores(self.reward, trajs)):  # one batched scoring
            ok = bool(r.passed)
            passed += ok
            malformed += ("error" in r.info) or (r.info.get("predicted", "x") is None)
            total += r.value
            per_item.append({"prompt": task.prompt[:80], "output": traj.response_text[:200], "reward": r.value,
                             "passed": ok})
        n = max(len(self.tasks), 1)
        return EvaluationResult(self.name, {"pass_rate": passed / n, "reward": total / n,
                                            "malformed_rate": malformed / n},
                                n_samples=len(self.tasks), per_item=per_item)


class AgentAccuracySuite:
    """Multi-turn tool-use accuracy and tool-use rate on tagged-answer tasks."""

    name = "agent_accuracy"

    def __init__(self, tasks: Sequence[Any], agent_engine, limit: Optional[int] = None):
        self.tasks = list(tasks)[: limit or None]
        self.engine = agent_engine

    @torch.no_grad()
    def run(self, policy=None, **kwargs: Any) -> EvaluationResult:
        from rl_project_b200.rollouts.agent import build_agent_prompt
        from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier

        verifier = TaggedAnswerVerifier()
        episodes = self.engine.run_episodes([build_agent_prompt(t.prompt) for t in self.tasks], temperature=0.0) \
            if self.tasks else []  # every task's episode advanced in lock-step
        outputs = [final for _, _, final in episodes]
        scores = verifier.verify_many(outputs, [t.answer for t in self.tasks])
        correct = sum(r.value >= 1.0 for r in scores)
        used_tool = sum("<tool_call>" in o for o in outputs)
        n = max(len(self.tasks), 1)
        return EvaluationResult(self.name, {"accuracy": correct / n, "tool_use_rate": used_tool / n},
                                n_samples=len(self.tasks))
