"""Evaluation results on disk: ``.jsonl`` (one result per line) or any other suffix (one JSON list), keyed
by the ``EvaluationResult.to_dict`` fields."""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Callable, Dict, Iterable, List

from rl_project_b200.core.protocols import EvaluationResult

_ENCODE: Dict[bool, Callable[[List[dict]], str]] = {
    True: lambda rows: "".join(json.dumps(r, default=str) + "\n" for r in rows),
    False: lambda rows: json.dumps(rows, indent=2, default=str),
}
_DECODE: Dict[bool, Callable[[str], List[Any]]] = {
    True: lambda text: [json.loads(line) for line in text.splitlines() if line.strip()],
    False: json.loads,
}


def _lines(path: Path) -> bool:
    return path.suffix == ".jsonl"


def save_results(results: Iterable[EvaluationResult], path: str | Path) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(_ENCODE[_lines(path)]([r.to_dict() for r in results]))
    return path


def _from_row(row: Dict[str, Any]) -> EvaluationResult:
    return EvaluationResult(suite=row["suite"], metrics=row["metrics"], n_samples=row.get("n_samples", 0),
                            details=row.get("details", {}), per_item=row.get("per_item", []))


def load_results(path: str | Path) -> List[EvaluationResult]:
    path = Path(path)
    return [_from_row(row) for row in _DECODE[_lines(path)](path.read_text())]


def merge_metrics(results: Iterable[EvaluationResult]) -> Dict[str, float]:
    """One flat ``{"suite/metric": value}`` mapping (the input of promotion gates)."""
    return {f"{r.suite}/{name}": value for r in results for name, value in r.metrics.items()}
