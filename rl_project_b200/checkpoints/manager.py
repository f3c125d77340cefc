"""Atomic, manifest-checked directory checkpoints.

On-disk format (kept byte-compatible with the reference contract so existing
checkpoints load; the reference package itself is absent from its snapshot and
its API is reconstructed from the call sites, e.g.
``src/forgeline/training/common/trainer.py:255-325`` and
``tests/unit/test_checkpoints.py``)::

    <root>/<name>/manifest.json   {format_version, created_at, step, algorithm, model_spec,
                                   tokenizer_meta, metadata, files{name: {size}}, complete}
    <root>/<name>/model.pt        model/adapter/value-head state
    <root>/<name>/optimizer.pt | scaler.pt | rng.pt | trainer.pt | experiment.json   (optional)
    <root>/LATEST                 name of the newest complete checkpoint

Writes go to ``<name>.tmp`` and are published with ``os.replace``.  Extension:
sharded runs (FSDP / TP / EP) add ``model.rank{r}.pt`` / ``optimizer.rank{r}.pt``
and a ``shard_layout`` manifest entry, written by every rank into the same
``.tmp`` directory before rank 0 publishes it.
"""

from __future__ import annotations

import json
import os
import shutil
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Mapping, Optional

import torch

from rl_project_b200.core.errors import (
    CheckpointCorruptError,
    CheckpointMismatchError,
    CheckpointNotFoundError,
    IncompatibleStateError,
)

FORMAT_VERSION = 1
_OPTIONAL = {
    "optimizer_state": "optimizer.pt",
    "scheduler_state": "scheduler.pt",
    "scaler_state": "scaler.pt",
    "rng_state": "rng.pt",
    "trainer_state": "trainer.pt",
}


@dataclass
class CheckpointState:
    model_state: Dict[str, Any]
    step: int = 0
    algorithm: str = ""
    model_spec: Dict[str, Any] = field(default_factory=dict)
    optimizer_state: Optional[Dict[str, Any]] = None
    scheduler_state: Optional[Dict[str, Any]] = None
    scaler_state: Optional[Dict[str, Any]] = None
    rng_state: Optional[Dict[str, Any]] = None
    trainer_state: Dict[str, Any] = field(default_factory=dict)
    tokenizer_meta: Optional[Dict[str, Any]] = None
    experiment: Optional[Dict[str, Any]] = None
    metadata: Dict[str, Any] = field(default_factory=dict)
    shards: Optional[Dict[str, Any]] = None  # {"model": [state per rank], "optimizer": [...], "layout": {...}}


def _to_cpu(obj: Any) -> Any:
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _to_cpu(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_cpu(v) for v in obj)
    return obj


def _fsync_dir(path: Path) -> None:
    try:
        fd = os.open(str(path), os.O_RDONLY)
        try:
            os.fsync(fd)
        finally:
            os.close(fd)
    except OSError:
        pass


class CheckpointManager:
    def __init__(self, root: str | os.PathLike, keep_last: int = 3, async_save: bool = False):
        self.root = Path(root)
        self.keep_last = keep_last
        self.async_save = async_save
        self._thread: Optional[threading.Thread] = None
        self._error: Optional[BaseException] = None

    # ----------------------------------------------------------------- save
    def save(self, state: CheckpointState, name: Optional[str] = None, is_best: bool = False) -> Path:
        name = name or f"step_{state.step:08d}"
        final = self.root / name
        snapshot = CheckpointState(**{k: _to_cpu(getattr(state, k)) for k in state.__dataclass_fields__})
        self.wait()
        if self.async_save:
            self._thread = threading.Thread(target=self._save_guarded, args=(snapshot, name, is_best), daemon=True)
            self._thread.start()
        else:
            self._write(snapshot, name, is_best)
        return final

    def _save_guarded(self, state: CheckpointState, name: str, is_best: bool) -> None:
        try:
            self._write(state, name, is_best)
        except BaseException as exc:  # surfaced by wait()
            self._error = exc

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            err, self._error = self._error, None
            raise err

    def _write(self, state: CheckpointState, name: str, is_best: bool) -> None:
        self.root.mkdir(parents=True, exist_ok=True)
        tmp = self.root / f"{name}.tmp"
        if tmp.exists():
            shutil.rmtree(tmp)
        tmp.mkdir(parents=True)
        files: Dict[str, Dict[str, int]] = {}

        def put(obj: Any, fname: str) -> None:
            torch.save(obj, tmp / fname)
            files[fname] = {"size": (tmp / fname).stat().st_size}

        put(state.model_state, "model.pt")
        for attr, fname in _OPTIONAL.items():
            val = getattr(state, attr)
            if val:
                put(val, fname)
        layout = None
        if state.shards:
            for kind in ("model", "optimizer"):
                for r, part in enumerate(state.shards.get(kind, []) or []):
                    put(part, f"{kind}.rank{r}.pt")
            layout = state.shards.get("layout")
        if state.experiment is not None:
            (tmp / "experiment.json").write_text(json.dumps(state.experiment, indent=2, default=str))
            files["experiment.json"] = {"size": (tmp / "experiment.json").stat().st_size}
        manifest = {
            "format_version": FORMAT_VERSION,
            "created_at": time.time(),
            "step": int(state.step),
            "algorithm": state.algorithm,
            "model_spec": state.model_spec,
            "tokenizer_meta": state.tokenizer_meta,
            "metadata": state.metadata,
            "files": files,
            "complete": True,
        }
        if layout is not None:
            manifest["shard_layout"] = layout
        (tmp / "manifest.json").write_text(json.dumps(manifest, indent=2, default=str))
        _fsync_dir(tmp)
        final = self.root / name
        if final.exists():
            shutil.rmtree(final)
        os.replace(tmp, final)
        _fsync_dir(self.root)
        if name != "best":
            (self.root / "LATEST.tmp").write_text(name)
            os.replace(self.root / "LATEST.tmp", self.root / "LATEST")
        if is_best and name != "best":
            best = self.root / "best"
            if best.exists():
                shutil.rmtree(best)
            shutil.copytree(final, best)
        self._rotate()

    def _rotate(self) -> None:
        steps = sorted(p for p in self.root.glob("step_*") if p.is_dir() and not p.name.endswith(".tmp"))
        for old in steps[: max(0, len(steps) - self.keep_last)]:
            shutil.rmtree(old, ignore_errors=True)

    # ----------------------------------------------------------------- discovery
    def list(self) -> List[Path]:
        if not self.root.exists():
            return []
        return sorted(p for p in self.root.iterdir() if p.is_dir() and not p.name.endswith(".tmp"))

    def find_latest(self) -> Optional[Path]:
        pointer = self.root / "LATEST"
        if pointer.exists():
            cand = self.root / pointer.read_text().strip()
            if cand.is_dir() and (cand / "manifest.json").exists():
                return cand
        best_step, best_path = -1, None
        for p in self.list():
            if p.name == "best":
                continue
            try:
                m = self.read_manifest(p)
            except Exception:
                continue
            if m.get("complete") and int(m.get("step", -1)) >= best_step:
                best_step, best_path = int(m["step"]), p
        return best_path

    # ----------------------------------------------------------------- load / validate
    @staticmethod
    def read_manifest(path: str | os.PathLike) -> Dict[str, Any]:
        path = Path(path)
        if not path.exists():
            raise CheckpointNotFoundError(f"checkpoint not found: {path}")
        mf = path / "manifest.json"
        if not mf.exists():
            raise CheckpointCorruptError(f"no manifest in {path}")
        try:
            data = json.loads(mf.read_text())
        except (json.JSONDecodeError, OSError) as exc:
            raise CheckpointCorruptError(f"unreadable manifest in {path}: {exc}") from exc
        if not isinstance(data, dict) or "files" not in data:
            raise CheckpointCorruptError(f"manifest in {path} is missing required keys")
        return data

    @staticmethod
    def validate(path: str | os.PathLike) -> Dict[str, Any]:
        path = Path(path)
        m = CheckpointManager.read_manifest(path)
        if not m.get("complete", False):
            raise CheckpointCorruptError(f"checkpoint {path} is incomplete")
        if int(m.get("format_version", 0)) > FORMAT_VERSION:
            raise CheckpointMismatchError(f"checkpoint {path} has newer format_version {m.get('format_version')}")
        if not (path / "model.pt").exists():
            raise CheckpointCorruptError(f"checkpoint {path} is missing model.pt")
        for fname, info in m["files"].items():
            f = path / fname
            if not f.exists():
                raise CheckpointCorruptError(f"checkpoint {path} is missing {fname}")
            if "size" in info and f.stat().st_size != int(info["size"]):
                raise CheckpointCorruptError(f"checkpoint file {fname} in {path} is truncated "
                                             f"({f.stat().st_size} != {info['size']} bytes)")
        return m

    @staticmethod
    def load(path: str | os.PathLike, map_location: Any = "cpu", expected_spec: Optional[Mapping[str, Any]] = None,
             expected_algorithm: Optional[str] = None, rank: Optional[int] = None) -> CheckpointState:
        path = Path(path)
        m = CheckpointManager.validate(path)
        if expected_spec:
            saved = m.get("model_spec") or {}
            diff = {k: (saved.get(k), v) for k, v in expected_spec.items() if k in saved and saved[k] != v}
            missing = [k for k in expected_spec if saved and k not in saved]
            if diff or (missing and len(missing) == len(expected_spec)):
                raise CheckpointMismatchError(f"model spec mismatch for {path}: {diff or missing}")
        if expected_algorithm and m.get("algorithm") and m["algorithm"] != expected_algorithm:
            raise CheckpointMismatchError(
                f"checkpoint {path} was written by {m['algorithm']!r}, expected {expected_algorithm!r}")

        def get(fname: str) -> Any:
            f = path / fname
            if not f.exists():
                return None
            try:
                return torch.load(f, map_location=map_location, weights_only=False)
            except Exception as exc:
                raise CheckpointCorruptError(f"cannot read {fname} in {path}: {exc}") from exc

        state = CheckpointState(model_state=get("model.pt"), step=int(m.get("step", 0)),
                                algorithm=m.get("algorithm", ""), model_spec=m.get("model_spec") or {},
                                tokenizer_meta=m.get("tokenizer_meta"), metadata=m.get("metadata") or {})
        for attr, fname in _OPTIONAL.items():
            val = get(fname)
            if val is not None:
                setattr(state, attr, val)
        if state.trainer_state is None:
            state.trainer_state = {}
        exp = path / "experiment.json"
        if exp.exists():
            state.experiment = json.loads(exp.read_text())
        if "shard_layout" in m:
            ranks = [rank] if rank is not None else range(int(m["shard_layout"].get("world_size", 0)))
            state.shards = {"layout": m["shard_layout"],
                            "model": {r: get(f"model.rank{r}.pt") for r in ranks},
                            "optimizer": {r: get(f"optimizer.rank{r}.pt") for r in ranks}}
        return state


def _strip_compile_prefix(state: Mapping[str, Any]) -> Dict[str, Any]:
    return {k.replace("_orig_mod.", ""): v for k, v in state.items()}


def load_model_state(model: torch.nn.Module, state: Mapping[str, Any], strict: bool = True):
    """Load ``state`` into ``model`` (``_orig_mod.`` prefixes stripped); shape mismatch -> IncompatibleStateError."""
    state = _strip_compile_prefix(state)
    own = model.state_dict()
    bad = {k: (tuple(v.shape), tuple(own[k].shape)) for k, v in state.items()
           if k in own and isinstance(v, torch.Tensor) and tuple(v.shape) != tuple(own[k].shape)}
    if bad:
        raise IncompatibleStateError(f"state shapes do not match the model: {dict(list(bad.items())[:5])}")
    try:
        return model.load_state_dict(state, strict=strict)
    except RuntimeError as exc:
        raise IncompatibleStateError(str(exc)) from exc
