"""Self-taught reasoning (``src/forgeline/training/star.py`` capabilities):
``STaRTrainer`` (rejection-sample correct rationales, SFT on them, repeat) and
``HillClimber`` (rejection-sample good tool-use trajectories into the task
set, then agent-GRPO rounds through the Trainer; checkpoint on improvement)."""

from __future__ import annotations

import json
import re
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence

import torch

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.core.protocols import GenerationSettings
from rl_project_b200.data.records import VerifiableTask, write_jsonl
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.rollouts.agent import AgentRolloutConfig, AgentRolloutEngine, build_agent_prompt
from rl_project_b200.rollouts.tools.parser import parse_tagged_output
from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier, extract_final_answer

log = get_logger("star")
_ANS = re.compile(r"<answer>\s*([\d,.\-]+)\s*</answer>", re.IGNORECASE)
_NUM = re.compile(r"-?\d+(?:,\d{3})*(?:\.\d+)?")


def star_prompt(problem: str) -> str:
    return ("Work through the problem one calculation at a time.\n"
            f"Finish with <answer>NUMBER</answer>\nProblem: {problem}\nSolution:")


def extract_star_answer(text: str) -> Optional[str]:
    m = _ANS.search(text)
    if m:
        return m.group(1).strip().replace(",", "")
    nums = _NUM.findall(text)
    return nums[-1].replace(",", "") if nums else None


def answers_match(pred: Optional[str], gt: str) -> bool:
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


class STaRTrainer:
    def __init__(self, policy, tasks: Sequence[VerifiableTask], cfg: STaRConfig, output_dir: str | Path):
        if len(tasks) < 2:
            raise ConfigError("STaR needs at least two tasks (train + eval)")
        self.policy, self.cfg = policy, cfg
        rows = list(tasks)
        n_eval = max(1, int(len(rows) * cfg.eval_fraction))
        self.eval_set, self.train_set = rows[-n_eval:], rows[: cfg.num_problems]
        self.out = Path(output_dir)
        self.out.mkdir(parents=True, exist_ok=True)
        self.optimizer = torch.optim.AdamW(policy.trainable_parameters(), lr=cfg.learning_rate)
        self.history: List[Dict[str, Any]] = []

    def _generate(self, prompt: str, temperature: float) -> str:
        ids = torch.tensor(self.policy.encode(prompt), dtype=torch.long)[None]
        with torch.no_grad():
            out = self.policy.generate(ids.to(self.policy.device), GenerationSettings(
                max_new_tokens=self.cfg.max_new_tokens, temperature=temperature,
                top_p=0.95 if temperature > 0 else None))
        return self.policy.decode(out[0])

    def generate_rationales(self) -> List[Dict[str, str]]:
        keep = []
        for task in self.train_set:
            prompt = star_prompt(task.prompt)
            for _ in range(self.cfg.samples_per_problem):
                r = self._generate(prompt, self.cfg.temperature)
                if answers_match(extract_star_answer(r), task.answer or ""):
                    keep.append({"prompt": prompt, "rationale": r, "answer": task.answer or ""})
        return keep

    def sft_on_rationales(self, examples: List[Dict[str, str]]) -> float:
        tot, n = 0.0, 0
        self.policy.train()
        block = getattr(self.policy.spec, "block_size", None)
        for _ in range(self.cfg.sft_epochs):
            for ex in examples:
                r = self.policy.encode(ex["rationale"])
                if not r:
                    continue
                q = torch.tensor(self.policy.encode(ex["prompt"]))[None]
                rr = torch.tensor(r)[None]
                if block is not None and q.shape[1] + rr.shape[1] > block:
                    q = q[:, -(block - rr.shape[1]):] if block > rr.shape[1] else q[:, -1:]
                    rr = rr[:, : block - q.shape[1]]
                loss = -self.policy.logprobs(q, rr).float().mean()
                loss.backward()
                torch.nn.utils.clip_grad_norm_(self.policy.trainable_parameters(), 1.0)
                self.optimizer.step()
                self.optimizer.zero_grad()
                tot += float(loss)
                n += 1
        self.policy.eval()
        return tot / max(n, 1)

    def evaluate(self) -> float:
        ok = sum(answers_match(extract_star_answer(self._generate(star_prompt(t.prompt), 0.0)), t.answer or "")
                 for t in self.eval_set)
        return ok / max(len(self.eval_set), 1)

    def run(self) -> Dict[str, Any]:
        base = self.evaluate()
        best = base
        self.history.append({"round": 0, "accuracy": round(base, 4), "correct_rationales": 0, "sft_loss": None})
        for rnd in range(1, self.cfg.num_rounds + 1):
            t0 = time.time()
            good = self.generate_rationales()
            yield_rate = len(good) / max(len(self.train_set) * self.cfg.samples_per_problem, 1)
            loss = self.sft_on_rationales(good) if good else None
            acc = self.evaluate()
            if acc > best:
                best = acc
                torch.save(self.policy.state_for_checkpoint(), self.out / "best_policy.pt")
            self.history.append({"round": rnd, "accuracy": round(acc, 4), "correct_rationales": len(good),
                                 "yield_rate": round(yield_rate, 4),
                                 "sft_loss": round(loss, 6) if loss is not None else None,
                                 "elapsed_s": round(time.time() - t0, 1)})
            log.info("star_round", round=rnd, accuracy=acc, correct=len(good))
        res = {"method": "star", "num_rounds": self.cfg.num_rounds, "baseline_acc": round(base, 4),
               "best_acc": round(best, 4), "improvement": round(best - base, 4), "history": self.history}
        (self.out / "star_results.json").write_text(json.dumps(res, indent=2))
        return res


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
        self.policy, self.cfg = policy, cfg
        rows = list(tasks)
        n_eval = min(cfg.eval_problems, max(1, len(rows) // 5))
        self.eval_set, self.train_set = rows[-n_eval:], rows[:-n_eval] or rows
        self.out = Path(output_dir)
        self.out.mkdir(parents=True, exist_ok=True)
        self.agent_cfg = agent_config or AgentRolloutConfig(max_new_tokens=cfg.max_new_tokens)
        self.engine = AgentRolloutEngine(policy, self.agent_cfg)
        self.verifier = TaggedAnswerVerifier()
        self.results: List[Dict[str, Any]] = []
        self.best_accuracy = 0.0

    def collect_rollouts(self) -> List[Dict[str, Any]]:
        kept = []
        for task in self.train_set:
            prompt = build_agent_prompt(task.prompt)
            cands = []
            for _ in range(self.cfg.rollouts_per_problem):
                _, _, out = self.engine.run_episode(prompt, temperature=0.9)
                r = self.verifier.verify(out, task.answer).value
                if r >= self.cfg.reward_threshold:
                    cands.append({"trajectory": out, "reward": r})
            cands.sort(key=lambda c: c["reward"], reverse=True)
            kept += [{"prompt": task.prompt, "answer": task.answer, "trajectory": c["trajectory"], "reward": c["reward"],
                      "tools": list(task.tools) or ["python_executor"]} for c in cands[: self.cfg.top_k_per_problem]]
        return kept

    def evaluate(self) -> Dict[str, float]:
        correct = tools = 0
        rewards = []
        for task in self.eval_set:
            _, _, out = self.engine.run_episode(build_agent_prompt(task.prompt), temperature=0.0)
            rewards.append(self.verifier.verify(out, task.answer).value)
            pred = extract_final_answer(out)
            correct += int(pred is not None and pred.strip() == (task.answer or "").strip())
            tools += int(parse_tagged_output(out).tool_call is not None)
        n = max(len(self.eval_set), 1)
        return {"accuracy": correct / n, "tool_use": tools / n, "avg_reward": sum(rewards) / n}

    def _grpo_round(self, tasks: Sequence[VerifiableTask], rnd: int) -> None:
        from rl_project_b200.core.config import ExperimentManifest, ModelSpec, OptimizerConfig, ScheduleConfig, TrainerConfig
        from rl_project_b200.core.lifecycle import RunContext
        from rl_project_b200.rollouts.rewards import build_reward_provider
        from rl_project_b200.training.common.trainer import Trainer
        from rl_project_b200.training.grpo import GRPOAlgorithm, GRPOConfig

        spec = self.policy.spec if isinstance(getattr(self.policy, "spec", None), ModelSpec) else ModelSpec()
        m = ExperimentManifest(name=f"hill_climb_round{rnd}", algorithm="grpo", model=spec,
                               output_dir=str(self.out / f"round_{rnd}"),
                               trainer=TrainerConfig(max_steps=self.cfg.grpo_steps_per_round, eval_every=0, log_every=10,
                                                     optimizer=OptimizerConfig(learning_rate=self.cfg.grpo_learning_rate,
                                                                               weight_decay=0.0),
                                                     schedule=ScheduleConfig(name="constant", warmup_steps=0)))
        ctx = RunContext.create(m, metrics_backend="local")
        alg = GRPOAlgorithm(self.policy, [t.to_dict() for t in tasks], build_reward_provider({"type": "tagged"}),
                            GRPOConfig(group_size=self.cfg.grpo_group_size, prompts_per_step=self.cfg.grpo_prompts_per_step,
                                       clip_ratio=self.cfg.grpo_clip, kl_coef=self.cfg.grpo_kl_coef, agent=True,
                                       seed=self.cfg.seed + rnd), agent_rollout=self.agent_cfg)
        Trainer(ctx, alg).fit()
        ctx.close()

    def run(self) -> List[Dict[str, Any]]:
        base = self.evaluate()
        self.best_accuracy = base["accuracy"]
        self.results.append({"round": 0, **base, "dataset_size": len(self.train_set)})
        for rnd in range(1, self.cfg.num_rounds + 1):
            t0 = time.time()
            extra = self.collect_rollouts()
            aug = list(self.train_set) + [VerifiableTask(prompt=r["prompt"], answer=r["answer"], task_type="tagged",
                                                         tools=r["tools"], meta={"trajectory": r["trajectory"]})
                                          for r in extra]
            write_jsonl(self.out / f"augmented_round{rnd}.jsonl", aug)
            self._grpo_round(aug, rnd)
            met = self.evaluate()
            if met["accuracy"] > self.best_accuracy:
                self.best_accuracy = met["accuracy"]
                torch.save(self.policy.state_for_checkpoint(), self.out / f"best_round_{rnd}.pt")
            self.results.append({"round": rnd, "dataset_size": len(aug), "added": len(extra),
                                 "elapsed_s": round(time.time() - t0, 1), **met})
            log.info("hill_climb_round", round=rnd, **met)
        (self.out / "hill_climb_results.json").write_text(json.dumps(self.results, indent=2))
        return self.results
