"""Critic rewards: a heuristic trajectory score in [0, 1], or a judge callable asked for one number
(the modes and scoring of ``src/forgeline/rollouts/rewards/critic.py``).

The heuristic is the sum of four components, each worth up to 0.25: a ``<final_answer>`` present;
reasoning keywords (0.25 for three or more, 0.10 for one or two); a ``<tool_call>``; and, for outputs of
at least 20 words, 4-gram diversity (0.25 above 0.8 distinct, 0.10 above 0.5).
"""

from __future__ import annotations

import re
from typing import Callable, List, Optional

from rl_project_b200.core.protocols import RewardResult, Trajectory

_KEYWORDS = frozenset({"because", "therefore", "first", "next", "then", "since", "step", "compute", "calculate",
                       "find", "let", "we"})
_FINAL = re.compile(r"<final_answer>(.*?)</final_answer>", re.DOTALL | re.IGNORECASE)
_CALL = re.compile(r"<tool_call>", re.IGNORECASE)


def _tiered(x: float, tiers) -> float:
    """Points of the first ``(threshold, points)`` tier that ``x`` exceeds (or reaches, for ``>=`` tiers)."""
    for ok, points in tiers:
        if ok(x):
            return points
    return 0.0


def _answer(output: str, words: List[str]) -> float:
    return 0.25 if _FINAL.search(output) else 0.0


def _reasoning(output: str, words: List[str]) -> float:
    hits = sum(w in _KEYWORDS for w in words)
    return _tiered(hits, ((lambda n: n >= 3, 0.25), (lambda n: n >= 1, 0.10)))


def _tool_use(output: str, words: List[str]) -> float:
    return 0.25 if _CALL.search(output) else 0.0


def _diversity(output: str, words: List[str]) -> float:
    if len(words) < 20:
        return 0.0
    grams = [tuple(words[i:i + 4]) for i in range(len(words) - 3)]
    distinct = len(set(grams)) / max(len(grams), 1)
    return _tiered(distinct, ((lambda r: r > 0.8, 0.25), (lambda r: r > 0.5, 0.10)))


_COMPONENTS = (_answer, _reasoning, _tool_use, _diversity)


def heuristic_critic_score(problem: str, output: str) -> float:
    words = output.lower().split()
    return round(min(sum(c(output, words) for c in _COMPONENTS), 1.0), 4)


_JUDGE_PROMPT = ("Rate this agent trajectory between 0.0 and 1.0 for: a final answer present, depth of reasoning, "
                 "sensible tool use and coherence.\nProblem: {problem}\nOutput:\n{output}\nReply with one number.")


class CriticReward:
    name = "critic"

    def __init__(self, mode: str = "heuristic", critic_fn: Optional[Callable[[str], str]] = None):
        if mode not in ("heuristic", "llm"):
            raise ValueError("mode must be heuristic|llm")
        if mode == "llm" and critic_fn is None:
            raise ValueError("mode='llm' requires critic_fn(prompt) -> str")
        self.mode, self.critic_fn = mode, critic_fn

    def _judge(self, problem: str, output: str) -> float:
        reply = (self.critic_fn(_JUDGE_PROMPT.format(problem=problem, output=output)) or "").strip()  # type: ignore[misc]
        m = re.search(r"\d+\.?\d*", reply)
        return min(max(float(m.group()), 0.0), 1.0) if m else 0.0

    def score(self, trajectory: Trajectory) -> RewardResult:
        problem = trajectory.task.get("prompt", trajectory.prompt_text)
        rate = heuristic_critic_score if self.mode == "heuristic" else self._judge
        return RewardResult(rate(problem, trajectory.response_text))
