"""Self-taught reasoning loops on batched generation (the capabilities of
``src/forgeline/training/star.py:1-260``).

``STaRTrainer``: each round samples rationales for the training problems, keeps those whose answer is
right (rejection sampling), fine-tunes on them and evaluates greedily on a held-out slice; the best
policy is saved.  ``HillClimber``: each round rejection-samples tool-using trajectories into the task set
and runs agent GRPO on the enlarged set through the Trainer; the policy is saved on improvement.

How the work is laid out differs from a per-sample loop:

* all ``problems x samples_per_problem`` rationales of a round come from ONE ``RolloutEngine.rollout_many``
  call (paged continuous batching on a GPU, length-grouped ``policy.generate`` batches elsewhere); the
  held-out problems are answered greedily the same way;
* the kept rationales are fine-tuned on in mini-batches of ``sft_batch_size`` rows of one prompt length
  (responses right-padded, loss = masked mean of the response log-probs), one optimizer step per
  mini-batch;
* the hill climber runs each round's ``problems x rollouts_per_problem`` agent episodes, and its
  evaluation episodes, as lock-step batches of ``AgentRolloutEngine.run_episodes``.
"""

from __future__ import annotations

import json
import re
import time
from collections import defaultdict
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.data.records import VerifiableTask, write_jsonl
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.rollouts.agent import AgentRolloutConfig, AgentRolloutEngine, build_agent_prompt
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine
from rl_project_b200.rollouts.tools.parser import parse_tagged_output
from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier, extract_final_answer

log = get_logger("star")

# a tagged answer wins; otherwise the last number in the text is the answer
_TAGGED = re.compile(r"<answer>\s*([\d,.\-]+)\s*</answer>", re.IGNORECASE)
_NUMBER = re.compile(r"-?\d+(?:,\d{3})*(?:\.\d+)?")


def star_prompt(problem: str) -> str:
    return ("Work through the problem one calculation at a time.\n"
            f"Finish with <answer>NUMBER</answer>\nProblem: {problem}\nSolution:")


def extract_star_answer(text: str) -> Optional[str]:
    tagged = _TAGGED.search(text)
    if tagged is not None:
        return tagged.group(1).strip().replace(",", "")
    numbers = _NUMBER.findall(text)
    return numbers[-1].replace(",", "") if numbers else None


def answers_match(pred: Optional[str], gt: str) -> bool:
    """Numeric equality within 1e-4 when both parse as numbers, else case-insensitive text equality."""
    if pred is None:
        return False
    try:
        return abs(float(pred) - float(gt.replace(",", ""))) < 1e-4
    except ValueError:
        return pred.strip().lower() == gt.strip().lower()


@dataclass
class STaRConfig:
    num_rounds: int = 3
    samples_per_problem: int = 8
    sft_epochs: int = 1
    learning_rate: float = 5e-6
    max_new_tokens: int = 256
    num_problems: int = 20
    temperature: float = 0.9
    eval_fraction: float = 0.1
    seed: int = 0
    sft_batch_size: int = 8


def _fit_block(q: List[int], r: List[int], block: Optional[int]) -> Tuple[List[int], List[int]]:
    """Trim a (prompt, response) pair to ``block`` tokens: the prompt loses its oldest tokens first (one is always
    kept), then the response its tail."""
    if block is None or len(q) + len(r) <= block:
        return q, r
    q = q[-(block - len(r)):] if block > len(r) else q[-1:]
    return q, r[: block - len(q)]


class STaRTrainer:
    def __init__(self, policy, tasks: Sequence[VerifiableTask], cfg: STaRConfig, output_dir: str | Path):
        if len(tasks) < 2:
            raise ConfigError("STaR needs at least two tasks (train + eval)")
        rows = list(tasks)
        held_out = max(1, int(len(rows) * cfg.eval_fraction))
        self.policy, self.cfg = policy, cfg
        self.train_set, self.eval_set = rows[: cfg.num_problems], rows[-held_out:]
        self.out = Path(output_dir)
        self.out.mkdir(parents=True, exist_ok=True)
        self.optimizer = torch.optim.AdamW(policy.trainable_parameters(), lr=cfg.learning_rate)
        self.history: List[Dict[str, Any]] = []

    def _engine(self, temperature: float) -> RolloutEngine:
        return RolloutEngine(self.policy, RolloutConfig(
            max_new_tokens=self.cfg.max_new_tokens, temperature=temperature,
            top_p=0.95 if temperature > 0 else None, record_old_logprobs=False,
            max_prompt_length=getattr(getattr(self.policy, "spec", None), "block_size", None) or 10**9))

    def _sample(self, problems: Sequence[VerifiableTask], n: int, temperature: float) -> List[List[str]]:
        """``n`` completions of the STaR prompt of every problem, from one batched rollout call."""
        prompts = [torch.tensor(self.policy.encode(star_prompt(t.prompt)), dtype=torch.long) for t in problems]
        groups = self._engine(temperature).rollout_many(prompts, group_size=n)
        return [[tr.response_text for tr in grp] for grp in groups]

    def generate_rationales(self) -> List[Dict[str, str]]:
        samples = self._sample(self.train_set, self.cfg.samples_per_problem, self.cfg.temperature)
        return [{"prompt": star_prompt(task.prompt), "rationale": text, "answer": task.answer or ""}
                for task, texts in zip(self.train_set, samples) for text in texts
                if answers_match(extract_star_answer(text), task.answer or "")]

    def _minibatches(self, examples: Sequence[Dict[str, str]]):
        """(prompt ids [B, Lq], response ids [B, Lr], response mask [B, Lr]) batches of one prompt length."""
        block = getattr(getattr(self.policy, "spec", None), "block_size", None)
        by_len: Dict[int, List[Tuple[List[int], List[int]]]] = defaultdict(list)
        for ex in examples:
            r = self.policy.encode(ex["rationale"])
            if r:
                q, r = _fit_block(self.policy.encode(ex["prompt"]), r, block)
                by_len[len(q)].append((q, r))
        pad = getattr(self.policy, "pad_token_id", 0)
        bs = max(1, self.cfg.sft_batch_size)
        for _, pairs in sorted(by_len.items()):
            for i in range(0, len(pairs), bs):
                chunk = pairs[i:i + bs]
                width = max(len(r) for _, r in chunk)
                resp = torch.full((len(chunk), width), pad, dtype=torch.long)
                mask = torch.zeros((len(chunk), width))
                for j, (_, r) in enumerate(chunk):
                    resp[j, : len(r)] = torch.tensor(r)
                    mask[j, : len(r)] = 1.0
                yield torch.tensor([q for q, _ in chunk], dtype=torch.long), resp, mask

    def sft_on_rationales(self, examples: List[Dict[str, str]]) -> float:
        """Fine-tune on the kept rationales; returns the mean mini-batch loss."""
        params = self.policy.trainable_parameters()
        losses: List[float] = []
        self.policy.train()
        for _ in range(self.cfg.sft_epochs):
            for q, r, mask in self._minibatches(examples):
                lp = self.policy.logprobs(q, r).float()
                m = mask.to(lp.device)
                loss = -(lp * m).sum() / m.sum().clamp_min(1.0)
                loss.backward()
                torch.nn.utils.clip_grad_norm_(params, 1.0)
                self.optimizer.step()
                self.optimizer.zero_grad(set_to_none=True)
                losses.append(float(loss))
        self.policy.eval()
        return sum(losses) / len(losses) if losses else 0.0

    def evaluate(self) -> float:
        answers = self._sample(self.eval_set, 1, 0.0)
        hits = [answers_match(extract_star_answer(texts[0]), t.answer or "") for t, texts in zip(self.eval_set, answers)]
        return sum(hits) / max(len(hits), 1)

    def run(self) -> Dict[str, Any]:
        baseline = best = self.evaluate()
        self.history.append({"round": 0, "accuracy": round(baseline, 4), "correct_rationales": 0, "sft_loss": None})
        attempts = max(len(self.train_set) * self.cfg.samples_per_problem, 1)
        for rnd in range(1, self.cfg.num_rounds + 1):
            started = time.time()
            kept = self.generate_rationales()
            loss = self.sft_on_rationales(kept) if kept else None
            acc = self.evaluate()
            if acc > best:
                best = acc
                torch.save(self.policy.state_for_checkpoint(), self.out / "best_policy.pt")
            self.history.append({"round": rnd, "accuracy": round(acc, 4), "correct_rationales": len(kept),
                                 "yield_rate": round(len(kept) / attempts, 4),
                                 "sft_loss": None if loss is None else round(loss, 6),
                                 "elapsed_s": round(time.time() - started, 1)})
            log.info("star_round", round=rnd, accuracy=acc, correct=len(kept))
        result = {"method": "star", "num_rounds": self.cfg.num_rounds, "baseline_acc": round(baseline, 4),
                  "best_acc": round(best, 4), "improvement": round(best - baseline, 4), "history": self.history}
        (self.out / "star_results.json").write_text(json.dumps(result, indent=2))
        return result


@dataclass
class HillClimbConfig:
    num_rounds: int = 5
    rollouts_per_problem: int = 4
    reward_threshold: float = 0.5
    top_k_per_problem: int = 2
    grpo_steps_per_round: int = 50
    grpo_group_size: int = 4
    grpo_learning_rate: float = 5e-6
    grpo_clip: float = 0.2
    grpo_kl_coef: float = 0.04
    grpo_prompts_per_step: int = 2
    max_new_tokens: int = 200
    eval_problems: int = 20
    seed: int = 42


class HillClimber:
    def __init__(self, policy, tasks: Sequence[VerifiableTask], cfg: HillClimbConfig, output_dir: str | Path,
                 agent_config: Optional[AgentRolloutConfig] = None):
        rows = list(tasks)
        held_out = min(cfg.eval_problems, max(1, len(rows) // 5))
        self.policy, self.cfg = policy, cfg
        self.eval_set, self.train_set = rows[-held_out:], rows[:-held_out] or rows
        self.out = Path(output_dir)
        self.out.mkdir(parents=True, exist_ok=True)
        self.agent_cfg = agent_config or AgentRolloutConfig(max_new_tokens=cfg.max_new_tokens)
        self.engine = AgentRolloutEngine(policy, self.agent_cfg)
        self.verifier = TaggedAnswerVerifier()
        self.results: List[Dict[str, Any]] = []
        self.best_accuracy = 0.0

    def collect_rollouts(self) -> List[Dict[str, Any]]:
        """The best ``top_k_per_problem`` episodes per training problem whose reward reaches the threshold."""
        k = self.cfg.rollouts_per_problem
        prompts = [build_agent_prompt(t.prompt) for t in self.train_set for _ in range(k)]
        episodes = self.engine.run_episodes(prompts, temperature=0.9)
        kept: List[Dict[str, Any]] = []
        for i, task in enumerate(self.train_set):
            scored = [(self.verifier.verify(final, task.answer).value, final) for _, _, final in episodes[i * k:(i + 1) * k]]
            good = sorted((s for s in scored if s[0] >= self.cfg.reward_threshold), key=lambda s: -s[0])
            kept += [{"prompt": task.prompt, "answer": task.answer, "trajectory": final, "reward": reward,
                      "tools": list(task.tools) or ["python_executor"]}
                     for reward, final in good[: self.cfg.top_k_per_problem]]
        return kept

    def evaluate(self) -> Dict[str, float]:
        episodes = self.engine.run_episodes([build_agent_prompt(t.prompt) for t in self.eval_set], temperature=0.0)
        n = max(len(self.eval_set), 1)
        correct = tool_use = 0
        reward = 0.0
        for task, (_, _, final) in zip(self.eval_set, episodes):
            reward += self.verifier.verify(final, task.answer).value
            pred = extract_final_answer(final)
            correct += int(pred is not None and pred.strip() == (task.answer or "").strip())
            tool_use += int(parse_tagged_output(final).tool_call is not None)
        return {"accuracy": correct / n, "tool_use": tool_use / n, "avg_reward": reward / n}

    def _grpo_round(self, tasks: Sequence[VerifiableTask], rnd: int) -> None:
        from rl_project_b200.core.config import ExperimentManifest, ModelSpec, OptimizerConfig, ScheduleConfig, TrainerConfig
        from rl_project_b200.core.lifecycle import RunContext
        from rl_project_b200.rollouts.rewards import build_reward_provider
        from rl_project_b200.training.common.trainer import Trainer
        from rl_project_b200.training.grpo import GRPOAlgorithm, GRPOConfig

        c = self.cfg
        spec = self.policy.spec if isinstance(getattr(self.policy, "spec", None), ModelSpec) else ModelSpec()
        trainer_cfg = TrainerConfig(max_steps=c.grpo_steps_per_round, eval_every=0, log_every=10,
                                    optimizer=OptimizerConfig(learning_rate=c.grpo_learning_rate, weight_decay=0.0),
                                    schedule=ScheduleConfig(name="constant", warmup_steps=0))
        manifest = ExperimentManifest(name=f"hill_climb_round{rnd}", algorithm="grpo", model=spec,
                                      output_dir=str(self.out / f"round_{rnd}"), trainer=trainer_cfg)
        grpo = GRPOConfig(group_size=c.grpo_group_size, prompts_per_step=c.grpo_prompts_per_step, clip_ratio=c.grpo_clip,
                          kl_coef=c.grpo_kl_coef, agent=True, seed=c.seed + rnd)
        ctx = RunContext.create(manifest, metrics_backend="local")
        alg = GRPOAlgorithm(self.policy, [t.to_dict() for t in tasks], build_reward_provider({"type": "tagged"}), grpo,
                            agent_rollout=self.agent_cfg)
        Trainer(ctx, alg).fit()
        ctx.close()

    def run(self) -> List[Dict[str, Any]]:
        first = self.evaluate()
        self.best_accuracy = first["accuracy"]
        self.results.append({"round": 0, **first, "dataset_size": len(self.train_set)})
        for rnd in range(1, self.cfg.num_rounds + 1):
            started = time.time()
            extra = self.collect_rollouts()
            enlarged = list(self.train_set) + [
                VerifiableTask(prompt=e["prompt"], answer=e["answer"], task_type="tagged", tools=e["tools"],
                               meta={"trajectory": e["trajectory"]}) for e in extra]
            write_jsonl(self.out / f"augmented_round{rnd}.jsonl", enlarged)
            self._grpo_round(enlarged, rnd)
            metrics = self.evaluate()
            if metrics["accuracy"] > self.best_accuracy:
                self.best_accuracy = metrics["accuracy"]
                torch.save(self.policy.state_for_checkpoint(), self.out / f"best_round_{rnd}.pt")
            self.results.append({"round": rnd, "dataset_size": len(enlarged), "added": len(extra),
                                 "elapsed_s": round(time.time() - started, 1), **metrics})
            log.info("hill_climb_round", round=rnd, **metrics)
        (self.out / "hill_climb_results.json").write_text(json.dumps(self.results, indent=2))
        return self.results
