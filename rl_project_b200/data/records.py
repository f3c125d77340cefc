"""Record schemas and validated JSONL IO.

Every dataset kind (supervised, preference, verifiable, process-reward, reward) is a dataclass whose
fields are described by a table of ``_Field`` specs: the JSON keys a value may come under (first match
wins), a coercion/validation function, and whether it is required.  One generic parser applies the table,
keeps the keys no field claimed in ``meta``, and runs the schema's cross-field check.  The schemas, their
key aliases and the JSONL conventions (``file:line`` in every error, ``on_error="skip"`` counting dropped
lines) are the data contract of the reference (``src/forgeline/data/records.py:22-225``), so existing
datasets load unchanged.
"""

from __future__ import annotations

import json
import math
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, Iterable, Iterator, List, Optional, Sequence, Tuple, Type, TypeVar

from rl_project_b200.core.errors import DatasetError, MalformedRecordError

T = TypeVar("T")
_MISSING = object()


# --------------------------------------------------------------------------- field coercions
def _nonempty_str(what: str) -> Callable[[Any], str]:
    def check(v: Any) -> str:
        if not isinstance(v, str) or not v:
            raise MalformedRecordError(what)
        return v
    return check


def _str(what: str) -> Callable[[Any], str]:
    def check(v: Any) -> str:
        if not isinstance(v, str):
            raise MalformedRecordError(what)
        return v
    return check


def _finite(what: str) -> Callable[[Any], float]:
    def check(v: Any) -> float:
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(float(v)):
            raise MalformedRecordError(what)
        return float(v)
    return check


def _list_of(item: Callable[[Any], Any], what: str) -> Callable[[Any], list]:
    def check(v: Any) -> list:
        if not isinstance(v, list):
            raise MalformedRecordError(what)
        return [item(x) for x in v]
    return check


def _as_text(v: Any) -> Optional[str]:
    return None if v is None else (v if isinstance(v, str) else str(v))


@dataclass(frozen=True)
class _Field:
    name: str
    keys: Tuple[str, ...]
    coerce: Callable[[Any], Any] = lambda v: v
    required: bool = True
    default: Any = None


def _parse(cls: Type[T], specs: Sequence[_Field], d: Dict[str, Any]) -> T:
    values: Dict[str, Any] = {}
    claimed = set()
    for spec in specs:
        claimed.update(spec.keys)
        raw = next((d[k] for k in spec.keys if k in d and d[k] is not None), _MISSING)
        if raw is _MISSING:
            if spec.required:
                spec.coerce(None)  # raises the field's message
            values[spec.name] = spec.default() if callable(spec.default) else spec.default
        else:
            values[spec.name] = spec.coerce(raw)
    values["meta"] = {k: v for k, v in d.items() if k not in claimed}
    rec = cls(**values)
    check = getattr(rec, "_check", None)
    if check is not None:
        check()
    return rec


def _emit(rec: Any, names: Sequence[str], skip_none: bool = False) -> Dict[str, Any]:
    out = {n: getattr(rec, n) for n in names if not (skip_none and getattr(rec, n) is None)}
    out.update(rec.meta)
    return out


# --------------------------------------------------------------------------- schemas
@dataclass
class SFTRecord:
    prompt: str
    response: str
    meta: Dict[str, Any] = field(default_factory=dict)

    _SPEC = (_Field("prompt", ("prompt",), _nonempty_str("SFT record needs a non-empty string 'prompt'")),
             _Field("response", ("response", "completion", "target"),
                    _nonempty_str("SFT record needs a non-empty string 'response'")))

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "SFTRecord":
        return _parse(cls, cls._SPEC, d)

    def to_dict(self) -> Dict[str, Any]:
        return _emit(self, ("prompt", "response"))


@dataclass
class PreferenceRecord:
    prompt: str
    chosen: str
    rejected: str
    meta: Dict[str, Any] = field(default_factory=dict)

    _SPEC = tuple(_Field(k, (k,), _str(f"preference record needs string field {k!r}"))
                  for k in ("prompt", "chosen", "rejected"))

    def _check(self) -> None:
        if self.chosen == self.rejected:
            raise MalformedRecordError("preference record has identical chosen and rejected responses")

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "PreferenceRecord":
        return _parse(cls, cls._SPEC, d)

    def to_dict(self) -> Dict[str, Any]:
        return _emit(self, ("prompt", "chosen", "rejected"))


@dataclass
class VerifiableTask:
    prompt: str
    answer: Optional[str] = None
    test_code: Optional[str] = None
    task_type: str = "math"
    tools: List[str] = field(default_factory=list)
    meta: Dict[str, Any] = field(default_factory=dict)

    _SPEC = (_Field("prompt", ("prompt", "problem", "question"),
                    _nonempty_str("verifiable task needs a non-empty 'prompt' (or 'problem')")),
             _Field("answer", ("answer",), _as_text, required=False),
             _Field("test_code", ("test_code", "test"), _as_text, required=False),
             _Field("task_type", ("task_type",), str, required=False),
             _Field("tools", ("available_tools", "tools"), _list_of(str, "'tools' must be a list"), required=False,
                    default=list))

    def _check(self) -> None:
        if self.answer is None and self.test_code is None:
            raise MalformedRecordError("verifiable task needs an 'answer' or 'test_code'")
        if self.task_type is None:  # code when only tests are given
            self.task_type = "code" if self.answer is None else "math"

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "VerifiableTask":
        return _parse(cls, cls._SPEC, d)

    def to_dict(self) -> Dict[str, Any]:
        return _emit(self, ("prompt", "task_type", "tools", "answer", "test_code"), skip_none=True)


@dataclass
class ProcessRecord:
    prompt: str
    steps: List[str]
    step_labels: List[float]
    answer: Optional[str] = None
    meta: Dict[str, Any] = field(default_factory=dict)

    _SHAPE = "process record needs 'prompt', list 'steps' and list 'step_labels'"
    _SPEC = (_Field("prompt", ("prompt",), _str(_SHAPE)),
             _Field("steps", ("steps",), _list_of(str, _SHAPE)),
             _Field("step_labels", ("step_labels",), _list_of(_finite("step labels must be finite numbers"), _SHAPE)),
             _Field("answer", ("answer",), required=False))

    def _check(self) -> None:
        if len(self.steps) != len(self.step_labels):
            raise MalformedRecordError("'steps' and 'step_labels' must have the same length")

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "ProcessRecord":
        return _parse(cls, cls._SPEC, d)


@dataclass
class RewardRecord:
    text: str
    score: float
    meta: Dict[str, Any] = field(default_factory=dict)

    _SHAPE = "reward record needs string 'text' and numeric 'score'"
    _SPEC = (_Field("text", ("text",), _str(_SHAPE)),
             _Field("score", ("score",), _finite("reward record score must be finite")))

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "RewardRecord":
        score = d.get("score")
        if isinstance(score, bool) or not isinstance(score, (int, float)):
            raise MalformedRecordError(cls._SHAPE)
        return _parse(cls, cls._SPEC, d)


SCHEMAS: Dict[str, Type[Any]] = {"supervised": SFTRecord, "preference": PreferenceRecord,
                                 "verifiable": VerifiableTask, "process": ProcessRecord, "reward": RewardRecord}


# --------------------------------------------------------------------------- JSONL
@dataclass
class ReadReport:
    read: int = 0
    skipped: int = 0
    errors: List[Tuple[int, str]] = field(default_factory=list)


def iter_jsonl(path: str | Path) -> Iterator[Tuple[int, Dict[str, Any]]]:
    """``(line number, object)`` for every non-blank line; a line that is not a JSON object raises with
    its ``file:line``."""
    path = Path(path)
    if not path.is_file():
        raise DatasetError(f"Dataset file not found: {path}")
    with path.open("r", encoding="utf-8") as fh:
        for lineno, raw in enumerate(fh, 1):
            if raw.isspace() or not raw:
                continue
            try:
                obj = json.loads(raw)
            except json.JSONDecodeError as exc:
                raise MalformedRecordError(f"{path}:{lineno}: invalid JSON ({exc.msg})") from None
            if type(obj) is not dict:
                raise MalformedRecordError(f"{path}:{lineno}: record must be a JSON object")
            yield lineno, obj


def read_jsonl(path: str | Path, schema: Type[T] | Callable[[Dict[str, Any]], T], *, on_error: str = "raise",
               report: Optional[ReadReport] = None) -> List[T]:
    """Parse every record of ``path`` with ``schema`` (a record class or a callable).  ``on_error="skip"``
    drops malformed records and lists them in ``report``."""
    if on_error not in ("raise", "skip"):
        raise DatasetError("on_error must be 'raise' or 'skip'")
    parse = getattr(schema, "from_dict", schema)
    rep = ReadReport() if report is None else report
    records: List[T] = []
    for lineno, obj in iter_jsonl(path):
        try:
            rec = parse(obj)
        except MalformedRecordError as exc:
            if on_error == "raise":
                raise MalformedRecordError(f"{path}:{lineno}: {exc.message}") from None
            rep.errors.append((lineno, exc.message))
            rep.skipped += 1
            continue
        records.append(rec)
        rep.read += 1
    return records


def write_jsonl(path: str | Path, records: Iterable[Any]) -> int:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    lines = [json.dumps(getattr(r, "to_dict", lambda r=r: r)(), ensure_ascii=False) for r in records]
    path.write_text("".join(line + "\n" for line in lines), encoding="utf-8")
    return len(lines)


def deterministic_split(items: List[T], val_fraction: float, seed: int) -> Tuple[List[T], List[T]]:
    """Seeded (train, val) partition: ``round(len * val_fraction)`` items drawn for validation (in draw
    order), the rest kept in their original order for training."""
    if not 0.0 <= val_fraction < 1.0:
        raise DatasetError("val_fraction must be in [0, 1)")
    rng = random.Random(seed)
    order = list(range(len(items)))
    rng.shuffle(order)
    n_val = int(round(len(items) * val_fraction))
    picked = order[:n_val]
    held = set(picked)
    return [x for i, x in enumerate(items) if i not in held], [items[i] for i in picked]
