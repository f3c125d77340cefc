"""Deterministic verifiers (``src/forgeline/rollouts/verifiers/__init__.py`` rules).

Each returns a ``RewardResult`` with ``passed`` and a value in [-1, 1]; any
exception inside a verifier becomes a failed result with the error recorded,
so one bad completion never aborts a rollout batch.  Scoring rules (answer
extraction order, partial credit, tag bonuses, code-test penalties) are the
reference's, because recorded rewards depend on them.

Added: ``last_token_parity`` -- 1 when the last generated token id is even
(the rule verifier of the GRPO benchmark configuration).
"""

from __future__ import annotations

import functools
import json
import re
from typing import Any, Optional, Tuple

from rl_project_b200.core.errors import VerifierError
from rl_project_b200.core.protocols import RewardResult
from rl_project_b200.core.registry import Registry
from rl_project_b200.rollouts.tools.python_executor import execute_python

VERIFIERS: Registry = Registry("verifier")


def _safe(fn):
    @functools.wraps(fn)
    def wrapper(self, output: str, target: Any = None) -> RewardResult:
        try:
            return fn(self, output, target)
        except Exception as exc:  # noqa: BLE001
            return RewardResult(value=0.0, passed=False, info={"error": f"{type(exc).__name__}: {exc}"})

    return wrapper


def _clean_num(s: str) -> str:
    return s.replace(",", "").replace("$", "").strip()


@VERIFIERS.register("math")
class MathVerifier:
    name = "math"

    def __init__(self, tolerance: float = 1e-6, partial_credit: bool = True):
        self.tolerance = tolerance
        self.partial_credit = partial_credit

    @staticmethod
    def extract_answer(text: str) -> Optional[str]:
        for pattern, flags in ((r"\\boxed\{([^}]+)\}", 0), (r"####\s*(.+?)(?:\n|$)", 0),
                               (r"(?:the\s+)?answer\s+is[:\s]*([^\n.]+)", re.IGNORECASE)):
            found = re.findall(pattern, text, flags)
            if found:
                return found[-1].strip()
        nums = re.findall(r"-?[\d,]+\.?\d*", text)
        return nums[-1].replace(",", "") if nums else None

    @_safe
    def verify(self, output: str, target: Any = None) -> RewardResult:
        if target is None:
            raise VerifierError("math verifier needs a target answer")
        pred = self.extract_answer(output)
        if pred is None:
            return RewardResult(0.0, passed=False, info={"predicted": None})
        pred, gold = _clean_num(pred), _clean_num(str(target))
        if pred.lower() == gold.lower():
            return RewardResult(1.0, passed=True, info={"predicted": pred})
        try:
            pv, gv = float(pred), float(gold)
        except ValueError:
            return RewardResult(0.0, passed=False, info={"predicted": pred})
        if abs(pv - gv) < self.tolerance:
            return RewardResult(1.0, passed=True, info={"predicted": pred})
        rel = abs(pv - gv) / max(abs(gv), 1e-8)
        value = 0.5 if (self.partial_credit and rel < 0.01) else 0.0
        return RewardResult(value, passed=False, info={"predicted": pred, "relative_error": rel})


@VERIFIERS.register("exact_match")
class ExactMatchVerifier:
    name = "exact_match"

    def __init__(self, normalize: bool = True):
        self.normalize = normalize

    @staticmethod
    def _norm(s: str) -> str:
        return re.sub(r"\s+", " ", s.strip().lower())

    @_safe
    def verify(self, output: str, target: Any = None) -> RewardResult:
        if target is None:
            raise VerifierError("exact_match verifier needs a target")
        a, b = (self._norm(output), self._norm(str(target))) if self.normalize else (output, str(target))
        return RewardResult(1.0 if a == b else 0.0, passed=a == b)


def normalize_answer(s: str) -> str:
    s = re.sub(r"\s+", " ", re.sub(r"[$,%]", "", s.strip().lower()))
    try:
        return str(float(s))
    except ValueError:
        return s


_FINAL = re.compile(r"<final_answer>(.*?)</final_answer>", re.DOTALL)


def extract_final_answer(text: str) -> Optional[str]:
    m = _FINAL.search(text)
    if m:
        return m.group(1).strip()
    nums = re.findall(r"(?<!\w)-?\d+(?:,\d{3})*(?:\.\d+)?(?!\w)", text)
    return nums[-1] if nums else None


@VERIFIERS.register("tagged_answer")
class TaggedAnswerVerifier:
    """1.0 for a correct ``<final_answer>``, ``tool_use_partial`` for a tool call that got a result, else 0."""

    name = "tagged_answer"

    def __init__(self, tool_use_partial: float = 0.1):
        self.tool_use_partial = tool_use_partial

    @_safe
    def verify(self, output: str, target: Any = None) -> RewardResult:
        if target is None:
            raise VerifierError("tagged_answer verifier needs a target")
        ans = extract_final_answer(output)
        if ans is not None and normalize_answer(ans) == normalize_answer(str(target)):
            return RewardResult(1.0, passed=True, info={"predicted": ans})
        if "<tool_call>" in output and "<tool_result>" in output:
            return RewardResult(self.tool_use_partial, passed=False, info={"predicted": ans, "tool_use": True})
        return RewardResult(0.0, passed=False, info={"predicted": ans})


def tag_format_reward(response: str) -> float:
    """0.02 for each of ``<think>``, ``<tool_call>``, ``<final_answer>`` present."""
    return 0.02 * sum(tag in response for tag in ("<think>", "<tool_call>", "<final_answer>"))


@VERIFIERS.register("code")
class CodeExecutionVerifier:
    name = "code"

    def __init__(self, timeout: float = 5.0, failure_penalty: float = -0.1):
        self.timeout = timeout
        self.failure_penalty = failure_penalty

    @staticmethod
    def extract_code(text: str) -> str:
        blocks = re.findall(r"```(?:python)?\s*\n(.*?)```", text, re.DOTALL)
        if blocks:
            return blocks[-1].strip()
        keep = [ln for ln in text.split("\n") if ln.startswith(("    ", "\t", "def ", "class "))]
        return "\n".join(keep) if keep else text

    @_safe
    def verify(self, output: str, target: Any = None) -> RewardResult:
        if not target:
            raise VerifierError("code verifier needs test code as the target")
        res = execute_python(self.extract_code(output) + "\n" + str(target), timeout=self.timeout)
        if not res.error:
            return RewardResult(1.0, passed=True)
        if "AssertionError" in res.stderr:
            return RewardResult(0.0, passed=False, info={"stderr": res.stderr[:200]})
        return RewardResult(self.failure_penalty, passed=False,
                            info={"stderr": res.stderr[:200], "timed_out": res.timed_out})


@VERIFIERS.register("format")
class FormatVerifier:
    name = "format"

    def __init__(self, format_spec: str = "cot"):
        if format_spec not in ("cot", "steps", "json"):
            raise VerifierError(f"unknown format_spec {format_spec!r}")
        self.format_spec = format_spec

    @_safe
    def verify(self, output: str, target: Any = None) -> RewardResult:
        spec = target or self.format_spec
        ok, score = {"cot": self._cot, "steps": self._steps}.get(spec, self._json)(output)
        return RewardResult(score, passed=ok)

    @staticmethod
    def _cot(text: str) -> Tuple[bool, float]:
        score = 0.0
        if "<think>" in text and "</think>" in text:
            score += 0.5
            m = re.search(r"<think>(.*?)</think>", text, re.DOTALL)
            if m and len(m.group(1).strip()) > 20:
                score += 0.3
        elif "think" in text.lower() or "let me" in text.lower():
            score += 0.2
        if "</think>" in text and len(text.split("</think>")[-1].strip()) > 5:
            score += 0.2
        return score >= 0.7, score

    @staticmethod
    def _steps(text: str) -> Tuple[bool, float]:
        n = len(re.findall(r"(?:step\s+\d|^\d+[.):])", text, re.IGNORECASE | re.MULTILINE))
        return n >= 2, min(n * 0.25, 1.0)

    @staticmethod
    def _json(text: str) -> Tuple[bool, float]:
        try:
            json.loads(text.strip())
            return True, 1.0
        except (json.JSONDecodeError, ValueError):
            m = re.search(r"\{.*\}", text, re.DOTALL)
            if m:
                try:
                    json.loads(m.group())
                    return True, 0.8
                except (json.JSONDecodeError, ValueError):
                    pass
            return False, 0.0


@VERIFIERS.register("last_token_parity")
class LastTokenParityVerifier:
    """1.0 when the last generated token id is even (token-level rule; ``target`` unused)."""

    name = "last_token_parity"

    @_safe
    def verify(self, output: Any, target: Any = None) -> RewardResult:
        ids = output.tolist() if hasattr(output, "tolist") else list(output)
        ok = bool(ids) and int(ids[-1]) % 2 == 0
        return RewardResult(1.0 if ok else 0.0, passed=ok)


def build_verifier(name: str, **kwargs: Any):
    return VERIFIERS.get(name)(**kwargs)
