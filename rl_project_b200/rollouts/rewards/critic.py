"""Critic rewards: a four-part heuristic score in [0, 1] or an LLM judge callable
(``src/forgeline/rollouts/rewards/critic.py`` scoring rules)."""

from __future__ import annotations

import re
from typing import Callable, Optional

from rl_project_b200.core.protocols import RewardResult, Trajectory

_KEYWORDS = {"because", "therefore", "first", "next", "then", "since", "step", "compute", "calculate", "find", "let", "we"}


def heuristic_critic_score(problem: str, output: str) -> float:
    words = output.lower().split()
    s = 0.25 if re.search(r"<final_answer>(.*?)</final_answer>", output, re.DOTALL | re.IGNORECASE) else 0.0
    kw = sum(w in _KEYWORDS for w in words)
    s += 0.25 if kw >= 3 else (0.10 if kw >= 1 else 0.0)
    if re.search(r"<tool_call>", output, re.IGNORECASE):
        s += 0.25
    if len(words) >= 20:
        grams = [" ".join(words[i:i + 4]) for i in range(len(words) - 3)]
        ratio = len(set(grams)) / max(len(grams), 1)
        s += 0.25 if ratio > 0.8 else (0.10 if ratio > 0.5 else 0.0)
    return round(min(s, 1.0), 4)


class CriticReward:
    name = "critic"

    def __init__(self, mode: str = "heuristic", critic_fn: Optional[Callable[[str], str]] = None):
        if mode not in ("heuristic", "llm"):
            raise ValueError("mode must be heuristic|llm")
        if mode == "llm" and critic_fn is None:
            raise ValueError("mode='llm' requires critic_fn(prompt) -> str")
        self.mode, self.critic_fn = mode, critic_fn

    def score(self, trajectory: Trajectory) -> RewardResult:
        problem = trajectory.task.get("prompt", trajectory.prompt_text)
        if self.mode == "heuristic":
            return RewardResult(heuristic_critic_score(problem, trajectory.response_text))
        ask = (f"Rate this agent trajectory between 0.0 and 1.0 for: a final answer present, depth of reasoning, "
               f"sensible tool use and coherence.\nProblem: {problem}\nOutput:\n{trajectory.response_text}\n"
               f"Reply with one number.")
        raw = (self.critic_fn(ask) or "").strip()  # type: ignore[misc]
        m = re.search(r"\d+\.?\d*", raw)
        return RewardResult(min(max(float(m.group()), 0.0), 1.0) if m else 0.0)
