"""Read-only views over what the framework writes to disk (the data layer of the dashboard).

Sources: run directories (``metrics.jsonl`` / ``events.jsonl`` of the local
metrics sink, the run's ``manifest.yaml``, checkpoint directories, evaluation
result files), the candidate registry JSON, and ``benchmarks/**/results.json``
evidence records -- the views of ``src/forgeline/dashboard/data.py``.  A tree is
walked once (``_Scan``) and every view reads from what that walk sorted out (run
directories, checkpoint directories, result files).  Everything is plain file
IO, testable and exportable without the HTTP server.
Checkpoints are loaded (``torch.load`` runs pickled code) only when they lie
under a configured runs root, never from an arbitrary request path.
"""

from __future__ import annotations

import hashlib
import json
import os
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional

MAX_POINTS = 1500
_SKIP = {".git", "__pycache__", "node_modules", ".venv", "site-packages"}
_NOT_RESULTS = {"manifest.json", "experiment.json", "metrics.jsonl", "events.jsonl"}


def _run_id(path: Path) -> str:
    return hashlib.sha1(str(path.resolve()).encode()).hexdigest()[:10]


def _read_jsonl(path: Path, limit: Optional[int] = None) -> List[Dict[str, Any]]:
    if not path.exists():
        return []
    rows = []
    with path.open() as fh:
        for line in fh:
            line = line.strip()
            if line:
                try:
                    rows.append(json.loads(line))
                except json.JSONDecodeError:
                    pass  # a half-written last line of a live run
    return rows[-limit:] if limit else rows


def _safe_json(path: Path) -> Dict[str, Any]:
    try:
        return json.loads(path.read_text())
    except Exception:  # noqa: BLE001
        return {}


@dataclass
class _Scan:
    """One walk of a directory tree, sorting what it finds: run directories (a metrics or events log),
    checkpoint directories (``manifest.json`` + ``model.pt``) and candidate evaluation-result files."""

    runs: List[Path] = field(default_factory=list)
    checkpoints: List[Path] = field(default_factory=list)
    result_files: List[Path] = field(default_factory=list)

    @classmethod
    def of(cls, root: Path, max_depth: int) -> "_Scan":
        scan = cls()
        if not root.exists():
            return scan
        top = root.resolve()
        base = len(top.parts)
        for dirpath, dirnames, filenames in os.walk(top):
            here = Path(dirpath)
            dirnames[:] = [] if len(here.parts) - base >= max_depth else \
                [d for d in dirnames if d not in _SKIP and not d.endswith(".tmp")]
            names = set(filenames)
            if names & {"metrics.jsonl", "events.jsonl"}:
                scan.runs.append(here)
            if {"manifest.json", "model.pt"} <= names:
                scan.checkpoints.append(here)
            scan.result_files += [here / n for n in sorted(names)
                                  if n.endswith((".json", ".jsonl")) and n not in _NOT_RESULTS]
        return scan


def downsample(points: List[List[float]], limit: int = MAX_POINTS) -> List[List[float]]:
    """At most ``limit`` evenly spaced points, always keeping the last one."""
    if len(points) <= limit:
        return points
    stride = len(points) / limit
    picked = [points[int(i * stride)] for i in range(limit - 1)]
    return picked + [points[-1]]


def _load_manifest(run_dir: Path) -> Dict[str, Any]:
    from rl_project_b200.core.config import load_config

    path = next((run_dir / n for n in ("manifest.yaml", "manifest.yml", "manifest.json") if (run_dir / n).exists()),
                None)
    if path is None:
        return {}
    try:
        return dict(load_config(path))
    except Exception:  # noqa: BLE001 - show the run even if its manifest no longer parses
        return {}


# event name -> run status, in precedence order
_STATUS = (("run.failed", "failed"), ("run.finished", "finished"), ("run.started", "running"))


def _status(events: List[Dict[str, Any]]) -> str:
    seen = {e.get("event") for e in events}
    return next((status for name, status in _STATUS if name in seen), "unknown")


def _run_row(d: Path) -> Dict[str, Any]:
    mpath, epath = d / "metrics.jsonl", d / "events.jsonl"
    events = _read_jsonl(epath)
    manifest = _load_manifest(d)
    last = _read_jsonl(mpath, limit=1)
    mtime = max((p.stat().st_mtime for p in (mpath, epath) if p.exists()), default=0.0)
    status = _status(events)
    algorithm = manifest.get("algorithm") or next((e["algorithm"] for e in events if e.get("algorithm")), "")
    return {"id": _run_id(d), "name": manifest.get("name") or d.name, "path": str(d), "algorithm": algorithm,
            "model_preset": manifest.get("model_preset", ""),
            "strategy": (manifest.get("distributed") or {}).get("strategy", ""),
            "orchestration": (manifest.get("orchestration") or {}).get("type", "local") if manifest else "",
            "status": status, "last_step": last[0].get("step") if last else None, "n_events": len(events),
            "updated_at": mtime, "live": status == "running" and time.time() - mtime < 120}


def discover_runs(roots: Iterable[str | Path], max_depth: int = 4) -> List[Dict[str, Any]]:
    """Every directory under the roots holding ``metrics.jsonl`` or ``events.jsonl``, newest first."""
    rows = {_run_id(d): _run_row(d) for root in map(Path, roots) for d in _Scan.of(root, max_depth).runs}
    return sorted(rows.values(), key=lambda r: r["updated_at"], reverse=True)


def _series(d: Path) -> Dict[str, List[List[float]]]:
    out: Dict[str, List[List[float]]] = {}
    for row in _read_jsonl(d / "metrics.jsonl"):
        for k, v in row.items():
            if k not in ("step", "ts") and isinstance(v, (int, float)) and not isinstance(v, bool):
                out.setdefault(k, []).append([row.get("step"), v])
    return {k: downsample(v) for k, v in sorted(out.items())}


def run_detail(run_dir: str | Path) -> Dict[str, Any]:
    d = Path(run_dir)
    events = _read_jsonl(d / "events.jsonl")
    scan = _Scan.of(d, 3)
    return {"id": _run_id(d), "path": str(d), "manifest": _load_manifest(d), "status": _status(events),
            "series": _series(d), "events": events[-500:],
            "summary": next((e for e in reversed(events) if e.get("event") == "run.finished"), None),
            "checkpoints": _checkpoint_rows(scan.checkpoints), "evaluations": _evaluation_rows(scan.result_files)}


def _checkpoint_row(d: Path) -> Dict[str, Any]:
    from rl_project_b200.checkpoints.manager import CheckpointManager

    try:
        manifest, valid, error = CheckpointManager.validate(d), True, ""
    except Exception as exc:  # noqa: BLE001
        manifest, valid, error = _safe_json(d / "manifest.json"), False, str(exc)
    latest = d.parent / "LATEST"
    spec, files = manifest.get("model_spec") or {}, manifest.get("files") or {}
    return {"path": str(d), "name": d.name, "step": manifest.get("step"), "algorithm": manifest.get("algorithm", ""),
            "created_at": manifest.get("created_at"), "valid": valid, "error": error,
            "size_bytes": sum(int(f.get("size", 0)) for f in files.values()), "files": sorted(files),
            "is_best": d.name == "best", "is_latest": latest.exists() and latest.read_text().strip() == d.name,
            "model": {k: spec[k] for k in ("n_layer", "n_head", "n_kv_head", "n_embd", "vocab_size", "block_size")
                      if k in spec}}


def _checkpoint_rows(dirs: Iterable[Path]) -> List[Dict[str, Any]]:
    return sorted((_checkpoint_row(d) for d in dirs), key=lambda c: (c["step"] is None, c["step"] or 0))


def list_checkpoints(root: str | Path, max_depth: int = 3) -> List[Dict[str, Any]]:
    return _checkpoint_rows(_Scan.of(Path(root), max_depth).checkpoints)


def _evaluation_rows(files: Iterable[Path]) -> List[Dict[str, Any]]:
    """Files that parse as evaluation results (``save_results``); anything else is skipped."""
    from rl_project_b200.evaluation.results import load_results

    out = []
    for p in files:
        if p.stat().st_size > 20_000_000:
            continue
        try:
            results = load_results(p)
        except Exception:  # noqa: BLE001 - not an evaluation file
            continue
        if results:
            out.append({"path": str(p), "results": [{"suite": r.suite, "metrics": r.metrics, "n_samples": r.n_samples,
                                                     "details": r.details} for r in results]})
    return out


def list_evaluations(root: str | Path, max_depth: int = 3) -> List[Dict[str, Any]]:
    """Result files written by ``save_results``."""
    return _evaluation_rows(_Scan.of(Path(root), max_depth).result_files)


def registry_view(path: str | Path) -> Dict[str, Any]:
    p = Path(path)
    if not p.exists():
        return {"path": str(p), "exists": False, "models": {}}
    from rl_project_b200.deployment.registry import CandidateRegistry

    models: Dict[str, List[Dict[str, Any]]] = {}
    for c in CandidateRegistry(p).list():
        models.setdefault(c.name, []).append(c.to_dict())
    return {"path": str(p), "exists": True, "models": models}


def benchmark_records(root: str | Path) -> List[Dict[str, Any]]:
    root = Path(root)
    if not root.exists():
        return []
    out = []
    for res in sorted(root.rglob("results.json")):
        data = _safe_json(res)
        summary = res.parent / "summary.md"
        out.append({"record": str(res.parent.relative_to(root)), "evidence": data.get("evidence", ""),
                    "revalidation_required": bool(data.get("revalidation_required", False)),
                    "revalidation_recommended": bool(data.get("revalidation_recommended", False)),
                    "published": data.get("published", True), "metrics": data.get("metrics", {}),
                    "notes": data.get("notes", []), "summary": summary.read_text() if summary.exists() else ""})
    return out


def inspect_checkpoint(path: str | Path, text: str = "", max_tokens: int = 48,
                       data_dir: Optional[str] = None) -> Dict[str, Any]:
    import torch

    from rl_project_b200.evaluation.inspection import (activation_flow, attention_patterns, layer_summary,
                                                       weight_statistics)
    from rl_project_b200.models.loading import load_model_from_checkpoint, resolve_tokenizer_for_checkpoint

    model, spec, state = load_model_from_checkpoint(path, "cpu")
    model = model.float().eval()
    stats = weight_statistics(model)
    out: Dict[str, Any] = {"checkpoint": str(path), "step": state.step, "algorithm": state.algorithm,
                           "spec": spec.to_dict(), "parameters": sum(s["numel"] for s in stats),
                           "layers": layer_summary(spec), "weights": stats}
    if text:
        try:
            tok = resolve_tokenizer_for_checkpoint(state, data_dir)
            ids = torch.tensor([tok.encode(text)[-max_tokens:]], dtype=torch.long)
            out["tokens"] = [tok.decode([i]) for i in ids[0].tolist()]
            out["attention"] = attention_patterns(model, ids, max_tokens=max_tokens)
            out["activations"] = activation_flow(model, ids)
        except Exception as exc:  # noqa: BLE001
            out["inspection_error"] = f"{type(exc).__name__}: {exc}"
    return out


@dataclass
class DashboardSources:
    runs: List[str] = field(default_factory=lambda: ["runs"])
    registry: str = "registry/candidates.json"
    benchmarks: str = "benchmarks"

    def checkpoint_allowed(self, path: str | Path) -> bool:
        """Only checkpoint directories under a configured runs root may be loaded."""
        target = Path(path).resolve()
        for root in self.runs:
            r = Path(root).resolve()
            if (r == target or r in target.parents) and (target / "manifest.json").exists():
                return True
        return False


def snapshot(sources: DashboardSources, include_runs_detail: bool = True) -> Dict[str, Any]:
    runs = discover_runs(sources.runs)
    return {"generated_at": time.time(),
            "sources": {"runs": sources.runs, "registry": sources.registry, "benchmarks": sources.benchmarks},
            "runs": runs, "run_details": {r["id"]: run_detail(r["path"]) for r in runs} if include_runs_detail else {},
            "registry": registry_view(sources.registry), "benchmarks": benchmark_records(sources.benchmarks)}
