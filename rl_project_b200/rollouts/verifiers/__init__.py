"""Deterministic verifiers: rule-based rewards for rollouts.

Every verifier maps ``(output, target)`` to a ``RewardResult`` (``passed`` and a value in [-1, 1]) and never
raises: an exception inside a rule becomes a failed result with the error recorded, so one malformed
completion cannot abort a batch.  The numeric rules -- which answer an extractor picks, partial credit,
format points, the code-failure penalty -- follow ``src/forgeline/rollouts/verifiers/__init__.py``
because recorded rewards depend on them; the structure here is its own:

* answers are pulled by an ordered list of extractors (first that finds something wins, the last match
  inside it);
* the ``cot`` format score is a table of (predicate, points) rows;
* every verifier has ``verify_many`` for a batch of outputs; the code verifier runs all of a batch's
  programs concurrently (one shared timeout) instead of one after another.

``last_token_parity`` (1 when the last generated token id is even) is the rule verifier of the GRPO
benchmark configuration.
"""

from __future__ import annotations

import json
import re
from typing import Any, Callable, List, Optional, Sequence, Tuple

from rl_project_b200.core.errors import VerifierError
from rl_project_b200.core.protocols import RewardResult
from rl_project_b200.core.registry import Registry
from rl_project_b200.rollouts.tools.python_executor import execute_many

VERIFIERS: Registry = Registry("verifier")


def _failed(exc: Exception) -> RewardResult:
    return RewardResult(value=0.0, passed=False, info={"error": f"{type(exc).__name__}: {exc}"})


class _Verifier:
    """Shared plumbing: ``verify`` guards ``_check``; ``verify_many`` maps it over a batch."""

    name = "base"
    needs_target = True

    def _check(self, output: Any, target: Any) -> RewardResult:
        raise NotImplementedError

    def verify(self, output: Any, target: Any = None) -> RewardResult:
        try:
            if self.needs_target and target is None:
                raise VerifierError(f"{self.name} verifier needs a target")
            return self._check(output, target)
        except Exception as exc:  # noqa: BLE001 - a bad completion scores as a failure
            return _failed(exc)

    def verify_many(self, outputs: Sequence[Any], targets: Sequence[Any]) -> List[RewardResult]:
        return [self.verify(o, t) for o, t in zip(outputs, targets)]


# ------------------------------------------------------------------ answers
def _last(pattern: str, flags: int = 0) -> Callable[[str], Optional[str]]:
    rx = re.compile(pattern, flags)

    def find(text: str) -> Optional[str]:
        hits = rx.findall(text)
        return hits[-1].strip() if hits else None

    return find


def _last_number(text: str) -> Optional[str]:
    hits = re.findall(r"-?[\d,]+\.?\d*", text)
    return hits[-1].replace(",", "") if hits else None


# boxed, then '#### x', then 'the answer is x', then the last number in the text
_MATH_EXTRACTORS = (_last(r"\\boxed\{([^}]+)\}"), _last(r"####\s*(.+?)(?:\n|$)"),
                    _last(r"(?:the\s+)?answer\s+is[:\s]*([^\n.]+)", re.IGNORECASE), _last_number)


def _first_found(extractors, text: str) -> Optional[str]:
    for ex in extractors:
        got = ex(text)
        if got is not None:
            return got
    return None


def _strip_number(s: str) -> str:
    return s.replace(",", "").replace("$", "").strip()


def _as_float(s: str) -> Optional[float]:
    try:
        return float(s)
    except ValueError:
        return None


@VERIFIERS.register("math")
class MathVerifier(_Verifier):
    """1 for the target answer (text-equal or numerically within ``tolerance``); 0.5 partial credit within 1 %
    relative error; else 0."""

    name = "math"

    def __init__(self, tolerance: float = 1e-6, partial_credit: bool = True):
        self.tolerance, self.partial_credit = tolerance, partial_credit

    @staticmethod
    def extract_answer(text: str) -> Optional[str]:
        return _first_found(_MATH_EXTRACTORS, text)

    def _check(self, output, target) -> RewardResult:
        raw = self.extract_answer(output)
        if raw is None:
            return RewardResult(0.0, passed=False, info={"predicted": None})
        pred, gold = _strip_number(raw), _strip_number(str(target))
        pv, gv = _as_float(pred), _as_float(gold)
        if pred.lower() == gold.lower() or (pv is not None and gv is not None and abs(pv - gv) < self.tolerance):
            return RewardResult(1.0, passed=True, info={"predicted": pred})
        if pv is None or gv is None:
            return RewardResult(0.0, passed=False, info={"predicted": pred})
        rel = abs(pv - gv) / max(abs(gv), 1e-8)
        return RewardResult(0.5 if self.partial_credit and rel < 0.01 else 0.0, passed=False,
                            info={"predicted": pred, "relative_error": rel})


@VERIFIERS.register("exact_match")
class ExactMatchVerifier(_Verifier):
    name = "exact_match"

    def __init__(self, normalize: bool = True):
        self.normalize = normalize

    @staticmethod
    def _norm(s: str) -> str:
        return " ".join(s.lower().split())

    def _check(self, output, target) -> RewardResult:
        f = self._norm if self.normalize else (lambda s: s)
        same = f(output) == f(str(target))
        return RewardResult(float(same), passed=same)


def normalize_answer(s: str) -> str:
    """Lower-cased, ``$ , %`` removed, whitespace collapsed; numbers in canonical float form."""
    s = re.sub(r"\s+", " ", re.sub(r"[$,%]", "", s.strip().lower()))
    f = _as_float(s)
    return str(f) if f is not None else s


def extract_final_answer(text: str) -> Optional[str]:
    """The ``<final_answer>`` body, else the last stand-alone number (thousands separators allowed)."""
    return _first_found((_first_tag("final_answer"),
                         _last(r"(?<!\w)-?\d+(?:,\d{3})*(?:\.\d+)?(?!\w)")), text)


def _first_tag(tag: str) -> Callable[[str], Optional[str]]:
    rx = re.compile(rf"<{tag}>(.*?)</{tag}>", re.DOTALL)
    return lambda text: (lambda m: m.group(1).strip() if m else None)(rx.search(text))


@VERIFIERS.register("tagged_answer")
class TaggedAnswerVerifier(_Verifier):
    """1 for a correct final answer; ``tool_use_partial`` when a tool was called and answered; else 0."""

    name = "tagged_answer"

    def __init__(self, tool_use_partial: float = 0.1):
        self.tool_use_partial = tool_use_partial

    def _check(self, output, target) -> RewardResult:
        ans = extract_final_answer(output)
        if ans is not None and normalize_answer(ans) == normalize_answer(str(target)):
            return RewardResult(1.0, passed=True, info={"predicted": ans})
        used_tool = "<tool_call>" in output and "<tool_result>" in output
        value = self.tool_use_partial if used_tool else 0.0
        info = {"predicted": ans, "tool_use": True} if used_tool else {"predicted": ans}
        return RewardResult(value, passed=False, info=info)


_FORMAT_TAGS = ("<think>", "<tool_call>", "<final_answer>")


def tag_format_reward(response: str) -> float:
    """0.02 for each of ``<think>``, ``<tool_call>``, ``<final_answer>`` present."""
    return 0.02 * sum(t in response for t in _FORMAT_TAGS)


# ------------------------------------------------------------------ code
@VERIFIERS.register("code")
class CodeExecutionVerifier(_Verifier):
    """Runs the completion's code followed by the target's test code: 1 if it exits cleanly, 0 on a failed
    assertion, ``failure_penalty`` for any other error or a timeout."""

    name = "code"
    needs_target = False  # checked per item (an empty test string is rejected too)

    def __init__(self, timeout: float = 5.0, failure_penalty: float = -0.1):
        self.timeout, self.failure_penalty = timeout, failure_penalty

    @staticmethod
    def extract_code(text: str) -> str:
        """The last fenced block, else the indented / ``def`` / ``class`` lines, else the whole text."""
        fenced = re.findall(r"```(?:python)?\s*\n(.*?)```", text, re.DOTALL)
        if fenced:
            return fenced[-1].strip()
        code_lines = [ln for ln in text.split("\n") if ln.startswith(("    ", "\t", "def ", "class "))]
        return "\n".join(code_lines) or text

    def _score(self, res) -> RewardResult:
        if not res.error:
            return RewardResult(1.0, passed=True)
        if "AssertionError" in res.stderr:
            return RewardResult(0.0, passed=False, info={"stderr": res.stderr[:200]})
        return RewardResult(self.failure_penalty, passed=False,
                            info={"stderr": res.stderr[:200], "timed_out": res.timed_out})

    def verify_many(self, outputs: Sequence[Any], targets: Sequence[Any]) -> List[RewardResult]:
        results: List[Optional[RewardResult]] = [None] * len(outputs)
        jobs: List[Tuple[int, str]] = []
        for i, (out, tgt) in enumerate(zip(outputs, targets)):
            try:
                if not tgt:
                    raise VerifierError("code verifier needs test code as the target")
                jobs.append((i, self.extract_code(out) + "\n" + str(tgt)))
            except Exception as exc:  # noqa: BLE001
                results[i] = _failed(exc)
        for (i, _), res in zip(jobs, execute_many([code for _, code in jobs], self.timeout)):
            results[i] = self._score(res)
        return results  # type: ignore[return-value]

    def _check(self, output, target) -> RewardResult:
        return self.verify_many([output], [target])[0]


# ------------------------------------------------------------------ format
def _think_body(text: str) -> str:
    m = re.search(r"<think>(.*?)</think>", text, re.DOTALL)
    return m.group(1).strip() if m else ""


def _has_think(t: str) -> bool:
    return "<think>" in t and "</think>" in t


# (predicate, points) rows of the chain-of-thought score; passes at 0.7
_COT_ROWS: Tuple[Tuple[Callable[[str], bool], float], ...] = (
    (_has_think, 0.5),
    (lambda t: _has_think(t) and len(_think_body(t)) > 20, 0.3),
    (lambda t: not _has_think(t) and ("think" in t.lower() or "let me" in t.lower()), 0.2),
    (lambda t: "</think>" in t and len(t.split("</think>")[-1].strip()) > 5, 0.2),
)


def _cot_score(text: str) -> Tuple[bool, float]:
    score = sum(points for pred, points in _COT_ROWS if pred(text))
    return score >= 0.7, score


def _steps_score(text: str) -> Tuple[bool, float]:
    n = len(re.findall(r"(?:step\s+\d|^\d+[.):])", text, re.IGNORECASE | re.MULTILINE))
    return n >= 2, min(0.25 * n, 1.0)


def _parses(s: str) -> bool:
    try:
        json.loads(s)
        return True
    except (json.JSONDecodeError, ValueError):
        return False


def _json_score(text: str) -> Tuple[bool, float]:
    if _parses(text.strip()):
        return True, 1.0
    m = re.search(r"\{.*\}", text, re.DOTALL)  # an embedded object earns less
    return (True, 0.8) if m and _parses(m.group()) else (False, 0.0)


_FORMATS = {"cot": _cot_score, "steps": _steps_score, "json": _json_score}


@VERIFIERS.register("format")
class FormatVerifier(_Verifier):
    name = "format"
    needs_target = False

    def __init__(self, format_spec: str = "cot"):
        if format_spec not in _FORMATS:
            raise VerifierError(f"unknown format_spec {format_spec!r}")
        self.format_spec = format_spec

    def _check(self, output, target) -> RewardResult:
        ok, score = _FORMATS.get(target or self.format_spec, _json_score)(output)
        return RewardResult(score, passed=ok)


@VERIFIERS.register("last_token_parity")
class LastTokenParityVerifier(_Verifier):
    """1 when the last generated token id is even (token-level rule; ``target`` unused)."""

    name = "last_token_parity"
    needs_target = False

    def _check(self, output, target) -> RewardResult:
        ids = output.tolist() if hasattr(output, "tolist") else list(output)
        even = bool(ids) and int(ids[-1]) % 2 == 0
        return RewardResult(float(even), passed=even)


def build_verifier(name: str, **kwargs: Any):
    return VERIFIERS.get(name)(**kwargs)
