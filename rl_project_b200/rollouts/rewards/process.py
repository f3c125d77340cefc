"""Process reward: discounted per-step credit plus the final-answer reward (the schedule and step
points of ``src/forgeline/rollouts/rewards/process.py``)::

    total = step_weight * sum_t gamma^(T-1-t) * r_t + final

with ``r_t`` = 0.15 for a verified computation or code that ran and printed, 0.10 for arithmetic that
parses, 0.05 for code that failed (or was not run), 0 otherwise, and ``final`` the tagged-answer
verifier's value.

How a step is judged: the first non-empty fenced code block decides if there is one; otherwise the first
assignment ``x = <arithmetic> [= <stated number>]`` whose right side evaluates (verified when the stated
number agrees to 1e-4 relative, merely parsed when nothing is stated; a disagreeing statement moves on to
the next assignment); otherwise any arithmetic run of at least four characters with an operator.
Arithmetic is evaluated from its ``ast`` (numbers, + - * / // % **, unary signs; exponents capped at 64),
never executed.  The discounted sum is accumulated backwards (Horner form).

Batched scoring (``ProcessReward.score_many``) gathers the code blocks of every step of every trajectory
and runs them concurrently against one timeout; the arithmetic rules need no execution.
"""

from __future__ import annotations

import ast
import operator
import re
from typing import Dict, List, Optional, Sequence, Tuple

from rl_project_b200.core.protocols import RewardResult, Trajectory
from rl_project_b200.rollouts.tools.python_executor import execute_many
from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier

STEP_REWARD_VERIFIED = 0.15
STEP_REWARD_PARSED = 0.10
STEP_REWARD_CODE_FAILED = 0.05
CODE_TIMEOUT_S = 3.0

_BOUNDARY = re.compile(r"\n\s*\n"  # blank line
                       r"|(?:^|\n)(?:Step\s+\d+[:\.]|#+\s)"  # 'Step 3:' or a markdown heading
                       r"|(?:^|\n)(?:First|Second|Third|Fourth|Next|Then|Finally)[,:\s]",  # ordinal openers
                       re.MULTILINE | re.IGNORECASE)
_FENCED = re.compile(r"```(?:python)?\s*(.*?)```", re.DOTALL)
_ASSIGNMENT = re.compile(r"([\w_]+)\s*=\s*(.+)")
_ARITH_RUN = re.compile(r"[-\d\s()+\-*/%^.]+")
_NUMBER = re.compile(r"-?\d+(?:,\d{3})*(?:\.\d+)?")
_ARITH_ONLY = re.compile(r"[-\d\s()+*/%.]+")

_BINARY = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul, ast.Div: operator.truediv,
           ast.FloorDiv: operator.floordiv, ast.Mod: operator.mod, ast.Pow: operator.pow}
_UNARY = {ast.USub: operator.neg, ast.UAdd: operator.pos}


def _value(node: ast.AST) -> float:
    if isinstance(node, ast.Expression):
        return _value(node.body)
    if isinstance(node, ast.Constant) and isinstance(node.value, (int, float)) and not isinstance(node.value, bool):
        return node.value
    if isinstance(node, ast.UnaryOp) and type(node.op) in _UNARY:
        return _UNARY[type(node.op)](_value(node.operand))
    if isinstance(node, ast.BinOp) and type(node.op) in _BINARY:
        left, right = _value(node.left), _value(node.right)
        if isinstance(node.op, ast.Pow) and abs(right) > 64:
            raise ValueError("exponent too large")
        return _BINARY[type(node.op)](left, right)
    raise ValueError("not arithmetic")


def safe_eval_arithmetic(expr: str) -> Optional[float]:
    """The value of an arithmetic expression (``,`` dropped, ``^`` read as ``**``), or None."""
    expr = expr.replace(",", "").replace("^", "**")
    if not _ARITH_ONLY.fullmatch(expr):
        return None
    try:
        v = float(_value(ast.parse(expr, mode="eval")))
    except Exception:  # noqa: BLE001 - syntax errors, division by zero, overflow
        return None
    return v if v == v and abs(v) != float("inf") else None


def parse_steps(response: str) -> List[str]:
    """Reasoning steps split at boundaries; a fragment under 25 characters joins the step before it."""
    steps: List[str] = []
    for piece in _BOUNDARY.split(response):
        piece = (piece or "").strip()
        if piece and steps and len(piece) < 25:
            steps[-1] = f"{steps[-1]} {piece}"
        elif piece:
            steps.append(piece)
    return steps or [response]


def _first_code(step: str) -> Optional[str]:
    return next((c.strip() for c in _FENCED.findall(step) if c.strip()), None)


def _stated_number(text: str) -> Optional[float]:
    nums = _NUMBER.findall(text)
    if not nums:
        return None
    try:
        return float(nums[0].replace(",", ""))
    except ValueError:
        return None


def _arithmetic_points(step: str) -> float:
    for m in _ASSIGNMENT.finditer(step):
        lhs_value, *stated = re.split(r"\s*=\s*(?=\d)", m.group(2).strip(), maxsplit=1)
        val = safe_eval_arithmetic(lhs_value.strip())
        if val is None:
            continue
        claim = _stated_number(stated[0]) if stated else None
        if claim is None:
            return STEP_REWARD_PARSED
        if abs(val - claim) < max(1e-4, abs(claim) * 1e-4):
            return STEP_REWARD_VERIFIED
    for m in _ARITH_RUN.finditer(step):
        expr = m.group(0).strip()
        if len(expr) >= 4 and any(op in expr for op in "+-*/") and safe_eval_arithmetic(expr) is not None:
            return STEP_REWARD_PARSED
    return 0.0


def _code_points(ran_ok: Optional[bool]) -> float:
    return STEP_REWARD_VERIFIED if ran_ok else STEP_REWARD_CODE_FAILED


def _score_steps(steps_per_item: Sequence[List[str]], execute_code: bool) -> List[List[float]]:
    """Step points of every item; all code blocks of the batch run concurrently."""
    points: List[List[float]] = [[0.0] * len(steps) for steps in steps_per_item]
    jobs: List[Tuple[int, int, str]] = []
    for i, steps in enumerate(steps_per_item):
        for j, step in enumerate(steps):
            code = _first_code(step)
            if code is None:
                points[i][j] = _arithmetic_points(step)
            elif execute_code:
                jobs.append((i, j, code))
            else:
                points[i][j] = _code_points(None)
    for (i, j, _), res in zip(jobs, execute_many([c for _, _, c in jobs], CODE_TIMEOUT_S)):
        points[i][j] = _code_points(not res.error and bool(res.stdout))
    return points


def score_step(step: str, execute_code: bool = True) -> float:
    return _score_steps([[step]], execute_code)[0][0]


def _discounted(points: Sequence[float], gamma: float) -> float:
    acc = 0.0
    for r in points:  # Horner: ((r0 * g + r1) * g + r2) ... = sum_t g^(T-1-t) r_t
        acc = acc * gamma + r
    return acc


def _combine(points: List[float], response: str, ground_truth: str, gamma: float,
             step_weight: float) -> Tuple[float, List[float]]:
    final = TaggedAnswerVerifier().verify(response, ground_truth).value
    return step_weight * _discounted(points, gamma) + final, points + [final]


def compute_process_reward(response: str, ground_truth: str, gamma: float = 0.9, step_weight: float = 1.0,
                           execute_code: bool = True) -> Tuple[float, List[float]]:
    """``(total, step points + [final])``."""
    points = _score_steps([parse_steps(response)], execute_code)[0]
    return _combine(points, response, ground_truth, gamma, step_weight)


class ProcessReward:
    name = "process"

    def __init__(self, gamma: float = 0.9, step_weight: float = 1.0, target_key: str = "answer",
                 execute_code: bool = True):
        self.gamma, self.step_weight, self.target_key, self.execute_code = gamma, step_weight, target_key, execute_code

    def _result(self, total: float, scores: List[float]) -> RewardResult:
        final = scores[-1]
        info: Dict[str, object] = {"step_scores": scores[:-1], "step_fraction": (total - final) / (total + 1e-8)}
        return RewardResult(total, passed=final >= 1.0, components={"step": total - final, "final": final}, info=info)

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        texts = [t.response_text for t in trajectories]
        points = _score_steps([parse_steps(x) for x in texts], self.execute_code)
        return [self._result(*_combine(p, x, str(t.task.get(self.target_key, "")), self.gamma, self.step_weight))
                for p, x, t in zip(points, texts, trajectories)]

    def score(self, trajectory: Trajectory) -> RewardResult:
        return self.score_many([trajectory])[0]
