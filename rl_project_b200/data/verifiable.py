"""Verifiable tasks (prompts with a checkable answer or tests) and plain RL prompt sets.

``VerifiableTaskDataset`` is a read-only sequence of ``VerifiableTask`` records with task-type views;
``load_prompts`` turns a prompt file (JSONL objects with ``prompt``/``text``, or plain lines) into token
id lists; ``extract_gsm8k_answer`` reads the ``#### <answer>`` line of a GSM8K solution.  Built-in tasks
and prompts match the reference's (``src/forgeline/data/verifiable.py``) so default runs are comparable.
"""

from __future__ import annotations

import json
from collections.abc import Sequence as _SequenceABC
from pathlib import Path
from typing import Iterator, List, Optional, Sequence

from rl_project_b200.core.errors import DatasetError, OptionalDependencyError
from rl_project_b200.data.records import ReadReport, VerifiableTask, read_jsonl, write_jsonl

_ARITHMETIC = (("What is 15 + 27?", "42"), ("What is 8 * 7?", "56"), ("What is 100 / 4?", "25"),
               ("What is 2^10?", "1024"), ("If x + 3 = 7, what is x?", "4"),
               ("What is the square root of 144?", "12"), ("What is 3! (3 factorial)?", "6"),
               ("What is 17 - 9?", "8"))
DEFAULT_ARITHMETIC_TASKS: List[VerifiableTask] = [VerifiableTask(prompt=q, answer=a) for q, a in _ARITHMETIC]
DEFAULT_PROMPTS: List[str] = ["Once upon a time", "The meaning of life is", "In a world where", "The key to success is"]


class VerifiableTaskDataset(_SequenceABC):
    kind = "verifiable"

    def __init__(self, tasks: Sequence[VerifiableTask]):
        self.tasks = list(tasks)
        if not self.tasks:
            raise DatasetError("verifiable task dataset is empty")

    @classmethod
    def from_jsonl(cls, path: str | Path, on_error: str = "raise", report: Optional[ReadReport] = None,
                   limit: Optional[int] = None) -> "VerifiableTaskDataset":
        tasks = read_jsonl(path, VerifiableTask, on_error=on_error, report=report)
        return cls(tasks if not limit else tasks[:limit])

    @classmethod
    def builtin_arithmetic(cls) -> "VerifiableTaskDataset":
        return cls(DEFAULT_ARITHMETIC_TASKS)

    def of_type(self, task_type: str) -> "VerifiableTaskDataset":
        """The tasks of one ``task_type`` (raises if there are none)."""
        return VerifiableTaskDataset([t for t in self.tasks if t.task_type == task_type])

    def __len__(self) -> int:
        return len(self.tasks)

    def __getitem__(self, i):
        return self.tasks[i]


def _prompt_texts(path: Path) -> Iterator[str]:
    with path.open(encoding="utf-8") as fh:
        for raw in fh:
            line = raw.strip()
            if not line:
                continue
            try:
                obj = json.loads(line)
            except json.JSONDecodeError:
                yield line
                continue
            yield (obj.get("prompt", obj.get("text", line)) if isinstance(obj, dict) else line)


def load_prompts(path: Optional[str | Path], tokenizer, max_length: int = 128) -> List[List[int]]:
    """Token ids of every prompt in ``path`` (cut to ``max_length``; empty ones dropped), or of the built-in
    prompts when ``path`` is unset or missing."""
    texts = _prompt_texts(Path(path)) if path and Path(path).exists() else iter(DEFAULT_PROMPTS)
    prompts = [ids[:max_length] for ids in map(tokenizer.encode, texts) if ids]
    if not prompts:
        raise DatasetError("no usable prompts found")
    return prompts


def extract_gsm8k_answer(solution: str) -> str:
    """The final answer of a GSM8K solution: the text after the last ``####`` marker, without commas or
    whitespace ("" when there is none)."""
    head, sep, tail = solution.rpartition("####")
    if not sep:
        return ""
    return "".join(ch for ch in tail.split("\n", 1)[0] if ch != "," and not ch.isspace())


def build_gsm8k_tool_dataset(output_path: str | Path, split: str = "train", limit: Optional[int] = None) -> int:
    """Write GSM8K as tagged-answer tool tasks (needs the optional ``datasets`` package and its cache)."""
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise OptionalDependencyError("datasets is not installed", hint="pip install datasets") from exc
    rows = load_dataset("openai/gsm8k", "main", split=split)
    if limit:
        rows = rows.select(range(min(limit, len(rows))))
    tasks = (VerifiableTask(prompt=r["question"], answer=a, task_type="tagged", tools=["python_executor"])
             for r in rows for a in [extract_gsm8k_answer(r["answer"])] if a)
    return write_jsonl(output_path, tasks)
