"""Process reward: discounted per-step credit plus the final-answer reward
(``src/forgeline/rollouts/rewards/process.py`` schedule:
``total = step_weight * sum_t gamma^(T-1-t) r_t + final``, with
r_t = 0.15 verified computation / running code, 0.10 parsable arithmetic,
0.05 code that failed)."""

from __future__ import annotations

import ast
import operator
import re
from typing import List, Optional, Tuple

from rl_project_b200.core.protocols import RewardResult, Trajectory
from rl_project_b200.rollouts.tools.python_executor import execute_python
from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier

_STEP_SEP = re.compile(r"\n\s*\n|(?:^|\n)(?:Step\s+\d+[:\.]|#+\s)|(?:^|\n)(?:First|Second|Third|Fourth|Next|Then|Finally)[,:\s]",
                       re.MULTILINE | re.IGNORECASE)
_CODE = re.compile(r"```(?:python)?\s*(.*?)```", re.DOTALL)
_ASSIGN = re.compile(r"([\w_]+)\s*=\s*(.+)")
_MATH = re.compile(r"[-\d\s()+\-*/%^.]+")
_NUM = re.compile(r"-?\d+(?:,\d{3})*(?:\.\d+)?")

STEP_REWARD_VERIFIED = 0.15
STEP_REWARD_PARSED = 0.10
STEP_REWARD_CODE_FAILED = 0.05

_OPS = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul, ast.Div: operator.truediv,
        ast.Mod: operator.mod, ast.Pow: operator.pow, ast.USub: operator.neg, ast.UAdd: operator.pos,
        ast.FloorDiv: operator.floordiv}


def _eval_node(n):
    if isinstance(n, ast.Expression):
        return _eval_node(n.body)
    if isinstance(n, ast.Constant) and isinstance(n.value, (int, float)):
        return n.value
    if isinstance(n, ast.BinOp) and type(n.op) in _OPS:
        a, b = _eval_node(n.left), _eval_node(n.right)
        if isinstance(n.op, ast.Pow) and abs(b) > 64:
            raise ValueError("exponent too large")
        return _OPS[type(n.op)](a, b)
    if isinstance(n, ast.UnaryOp) and type(n.op) in _OPS:
        return _OPS[type(n.op)](_eval_node(n.operand))
    raise ValueError("not arithmetic")


def safe_eval_arithmetic(expr: str) -> Optional[float]:
    """Arithmetic over + - * / % ** only (parsed with ``ast``, nothing executed); None otherwise."""
    expr = expr.replace(",", "").replace("^", "**")
    if not re.fullmatch(r"[-\d\s()+*/%.]+", expr):
        return None
    try:
        v = _eval_node(ast.parse(expr, mode="eval"))
    except Exception:
        return None
    if isinstance(v, (int, float)) and v == v and abs(v) != float("inf"):
        return float(v)
    return None


def parse_steps(response: str) -> List[str]:
    steps: List[str] = []
    for s in _STEP_SEP.split(response):
        s = (s or "").strip()
        if not s:
            continue
        if steps and len(s) < 25:
            steps[-1] += " " + s
        else:
            steps.append(s)
    return steps or [response]


def score_step(step: str, execute_code: bool = True) -> float:
    for code in _CODE.findall(step):
        code = code.strip()
        if not code:
            continue
        if not execute_code:
            return STEP_REWARD_CODE_FAILED
        res = execute_python(code, timeout=3.0)
        return STEP_REWARD_VERIFIED if (not res.error and res.stdout) else STEP_REWARD_CODE_FAILED
    for m in _ASSIGN.finditer(step):
        parts = re.split(r"\s*=\s*(?=\d)", m.group(2).strip(), maxsplit=1)
        val = safe_eval_arithmetic(parts[0].strip())
        if val is None:
            continue
        if len(parts) > 1:
            stated = _NUM.findall(parts[1])
            if stated:
                try:
                    s = float(stated[0].replace(",", ""))
                except ValueError:
                    s = None
                if s is not None:
                    if abs(val - s) < max(1e-4, abs(s) * 1e-4):
                        return STEP_REWARD_VERIFIED
                    continue
        return STEP_REWARD_PARSED
    for m in _MATH.finditer(step):
        expr = m.group(0).strip()
        if len(expr) >= 4 and any(op in expr for op in "+-*/") and safe_eval_arithmetic(expr) is not None:
            return STEP_REWARD_PARSED
    return 0.0


def compute_process_reward(response: str, ground_truth: str, gamma: float = 0.9, step_weight: float = 1.0,
                           execute_code: bool = True) -> Tuple[float, List[float]]:
    scores = [score_step(s, execute_code) for s in parse_steps(response)]
    T = len(scores)
    disc = step_weight * sum(gamma ** (T - 1 - t) * r for t, r in enumerate(scores))
    final = TaggedAnswerVerifier().verify(response, ground_truth).value
    return disc + final, scores + [final]


class ProcessReward:
    name = "process"

    def __init__(self, gamma: float = 0.9, step_weight: float = 1.0, target_key: str = "answer",
                 execute_code: bool = True):
        self.gamma, self.step_weight, self.target_key, self.execute_code = gamma, step_weight, target_key, execute_code

    def score(self, trajectory: Trajectory) -> RewardResult:
        total, scores = compute_process_reward(trajectory.response_text, str(trajectory.task.get(self.target_key, "")),
                                               self.gamma, self.step_weight, self.execute_code)
        final = scores[-1]
        return RewardResult(total, passed=final >= 1.0, components={"step": total - final, "final": final},
                            info={"step_scores": scores[:-1], "step_fraction": (total - final) / (total + 1e-8)})
