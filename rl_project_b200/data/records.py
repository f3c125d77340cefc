"""Record schemas and validated JSONL IO (``src/forgeline/data/records.py:22-225`` contract).

Each dataset kind has a small dataclass with ``from_dict`` validation;
``read_jsonl`` reports ``file:line`` for malformed records and either raises
``MalformedRecordError`` or, with ``on_error="skip"``, drops and counts them.
"""

from __future__ import annotations

import json
import math
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, Iterable, Iterator, List, Optional, Tuple, Type, TypeVar

from rl_project_b200.core.errors import DatasetError, MalformedRecordError

T = TypeVar("T")


def _extra(d: Dict[str, Any], used: Tuple[str, ...]) -> Dict[str, Any]:
    return {k: v for k, v in d.items() if k not in used}


@dataclass
class SFTRecord:
    prompt: str
    response: str
    meta: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "SFTRecord":
        prompt = d.get("prompt")
        response = d.get("response", d.get("completion", d.get("target")))
        if not isinstance(prompt, str) or not prompt:
            raise MalformedRecordError("SFT record needs a non-empty string 'prompt'")
        if not isinstance(response, str) or not response:
            raise MalformedRecordError("SFT record needs a non-empty string 'response'")
        return cls(prompt, response, _extra(d, ("prompt", "response", "completion", "target")))

    def to_dict(self) -> Dict[str, Any]:
        return {"prompt": self.prompt, "response": self.response, **self.meta}


@dataclass
class PreferenceRecord:
    prompt: str
    chosen: str
    rejected: str
    meta: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "PreferenceRecord":
        for key in ("prompt", "chosen", "rejected"):
            if not isinstance(d.get(key), str):
                raise MalformedRecordError(f"preference record needs string field {key!r}")
        if d["chosen"] == d["rejected"]:
            raise MalformedRecordError("preference record has identical chosen and rejected responses")
        return cls(d["prompt"], d["chosen"], d["rejected"], _extra(d, ("prompt", "chosen", "rejected")))

    def to_dict(self) -> Dict[str, Any]:
        return {"prompt": self.prompt, "chosen": self.chosen, "rejected": self.rejected, **self.meta}


@dataclass
class VerifiableTask:
    prompt: str
    answer: Optional[str] = None
    test_code: Optional[str] = None
    task_type: str = "math"
    tools: List[str] = field(default_factory=list)
    meta: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "VerifiableTask":
        prompt = d.get("prompt", d.get("problem", d.get("question")))
        if not isinstance(prompt, str) or not prompt:
            raise MalformedRecordError("verifiable task needs a non-empty 'prompt' (or 'problem')")
        answer = d.get("answer")
        test_code = d.get("test_code", d.get("test"))
        if answer is None and test_code is None:
            raise MalformedRecordError("verifiable task needs an 'answer' or 'test_code'")
        if answer is not None and not isinstance(answer, str):
            answer = str(answer)
        tools = d.get("available_tools", d.get("tools", [])) or []
        if not isinstance(tools, list):
            raise MalformedRecordError("'tools' must be a list")
        kind = d.get("task_type", "code" if test_code and answer is None else "math")
        used = ("prompt", "problem", "question", "answer", "test_code", "test", "available_tools", "tools", "task_type")
        return cls(prompt, answer, test_code, kind, list(tools), _extra(d, used))

    def to_dict(self) -> Dict[str, Any]:
        out: Dict[str, Any] = {"prompt": self.prompt, "task_type": self.task_type, "tools": list(self.tools)}
        if self.answer is not None:
            out["answer"] = self.answer
        if self.test_code is not None:
            out["test_code"] = self.test_code
        out.update(self.meta)
        return out


@dataclass
class ProcessRecord:
    prompt: str
    steps: List[str]
    step_labels: List[float]
    answer: Optional[str] = None
    meta: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "ProcessRecord":
        steps, labels = d.get("steps"), d.get("step_labels")
        if not isinstance(d.get("prompt"), str) or not isinstance(steps, list) or not isinstance(labels, list):
            raise MalformedRecordError("process record needs 'prompt', list 'steps' and list 'step_labels'")
        if len(steps) != len(labels):
            raise MalformedRecordError("'steps' and 'step_labels' must have the same length")
        if any(not isinstance(x, (int, float)) or not math.isfinite(float(x)) for x in labels):
            raise MalformedRecordError("step labels must be finite numbers")
        return cls(d["prompt"], [str(s) for s in steps], [float(x) for x in labels], d.get("answer"),
                   _extra(d, ("prompt", "steps", "step_labels", "answer")))


@dataclass
class RewardRecord:
    text: str
    score: float
    meta: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "RewardRecord":
        if not isinstance(d.get("text"), str) or not isinstance(d.get("score"), (int, float)):
            raise MalformedRecordError("reward record needs string 'text' and numeric 'score'")
        if not math.isfinite(float(d["score"])):
            raise MalformedRecordError("reward record score must be finite")
        return cls(d["text"], float(d["score"]), _extra(d, ("text", "score")))


SCHEMAS: Dict[str, Type[Any]] = {"supervised": SFTRecord, "preference": PreferenceRecord,
                                 "verifiable": VerifiableTask, "process": ProcessRecord, "reward": RewardRecord}


@dataclass
class ReadReport:
    read: int = 0
    skipped: int = 0
    errors: List[Tuple[int, str]] = field(default_factory=list)


def iter_jsonl(path: str | Path) -> Iterator[Tuple[int, Dict[str, Any]]]:
    path = Path(path)
    if not path.exists():
        raise DatasetError(f"Dataset file not found: {path}")
    with path.open("r", encoding="utf-8") as fh:
        for lineno, line in enumerate(fh, start=1):
            line = line.strip()
            if not line:
                continue
            try:
                obj = json.loads(line)
            except json.JSONDecodeError as exc:
                raise MalformedRecordError(f"{path}:{lineno}: invalid JSON ({exc.msg})") from None
            if not isinstance(obj, dict):
                raise MalformedRecordError(f"{path}:{lineno}: record must be a JSON object")
            yield lineno, obj


def read_jsonl(path: str | Path, schema: Type[T] | Callable[[Dict[str, Any]], T], *, on_error: str = "raise",
               report: Optional[ReadReport] = None) -> List[T]:
    if on_error not in ("raise", "skip"):
        raise DatasetError("on_error must be 'raise' or 'skip'")
    parse = schema.from_dict if hasattr(schema, "from_dict") else schema  # type: ignore[union-attr]
    rep = report if report is not None else ReadReport()
    out: List[T] = []
    for lineno, obj in iter_jsonl(path):
        try:
            out.append(parse(obj))
            rep.read += 1
        except MalformedRecordError as exc:
            if on_error == "raise":
                raise MalformedRecordError(f"{path}:{lineno}: {exc.message}") from None
            rep.skipped += 1
            rep.errors.append((lineno, exc.message))
    return out


def write_jsonl(path: str | Path, records: Iterable[Any]) -> int:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    n = 0
    with path.open("w", encoding="utf-8") as fh:
        for r in records:
            fh.write(json.dumps(r.to_dict() if hasattr(r, "to_dict") else r, ensure_ascii=False) + "\n")
            n += 1
    return n


def deterministic_split(items: List[T], val_fraction: float, seed: int) -> Tuple[List[T], List[T]]:
    if not 0.0 <= val_fraction < 1.0:
        raise DatasetError("val_fraction must be in [0, 1)")
    order = list(range(len(items)))
    random.Random(seed).shuffle(order)
    n_val = int(round(len(items) * val_fraction))
    val_set = set(order[:n_val])
    return [items[i] for i in range(len(items)) if i not in val_set], [items[i] for i in order[:n_val]]
