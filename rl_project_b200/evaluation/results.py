"""Evaluation results as JSON (list) or JSONL (one result per line)."""

from __future__ import annotations

import json
from pathlib import Path
from typing import Dict, Iterable, List

from rl_project_b200.core.protocols import EvaluationResult


def save_results(results: Iterable[EvaluationResult], path: str | Path) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    rows = [r.to_dict() for r in results]
    if path.suffix == ".jsonl":
        path.write_text("".join(json.dumps(r, default=str) + "\n" for r in rows))
    else:
        path.write_text(json.dumps(rows, indent=2, default=str))
    return path


def load_results(path: str | Path) -> List[EvaluationResult]:
    path = Path(path)
    text = path.read_text()
    rows = [json.loads(line) for line in text.splitlines() if line.strip()] if path.suffix == ".jsonl" \
        else json.loads(text)
    return [EvaluationResult(suite=r["suite"], metrics=r["metrics"], n_samples=r.get("n_samples", 0),
                             details=r.get("details", {}), per_item=r.get("per_item", [])) for r in rows]


def merge_metrics(results: Iterable[EvaluationResult]) -> Dict[str, float]:
    """One flat ``{"suite/metric": value}`` mapping (the input of promotion gates)."""
    return {f"{r.suite}/{k}": v for r in results for k, v in r.metrics.items()}
