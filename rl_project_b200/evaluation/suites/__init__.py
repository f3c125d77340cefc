"""Standard benchmarks with small built-in offline samples.

Each benchmark gives ``tasks()``, ``format_prompt(task, few_shot)`` and ``score(task, output)`` (the
interface of ``src/forgeline/evaluation/suites/__init__.py``).  What differs between benchmarks is data,
not code: a ``BenchmarkSpec`` in ``SPECS`` holds the samples, the public dataset and its row mapping, the
prompt and few-shot writers and the scorer, and one ``Benchmark`` class serves them all (the named
classes bind a spec).  With ``offline=False`` and the ``datasets`` package present, the public test sets
are loaded; otherwise the built-in samples (written for this project, for wiring and CI, not for reporting
scores) are used.  ``BenchmarkSuite`` decodes every task of a run in one batched rollout and scores the
run in one batch (the code benchmark runs all programs concurrently).
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch

from rl_project_b200.core.protocols import EvaluationResult
from rl_project_b200.core.registry import Registry
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.rollouts.tools.python_executor import execute_many

log = get_logger("forgeline.evaluation.suites")

BENCHMARKS: Registry = Registry("benchmark")


def _load_hf(name: str, split: str, **kwargs: Any):
    try:
        from datasets import load_dataset  # optional dependency

        return load_dataset(name, split=split, **kwargs)
    except Exception as exc:  # noqa: BLE001 - offline or not installed
        log.warning("hf_dataset_unavailable", dataset=name, error=str(exc)[:120])
        return None


# ------------------------------------------------------------------ built-in samples (written for this project)
MMLU_SAMPLES = [
    {"question": "How many bits are in one byte?", "choices": ["4", "8", "16", "32"], "answer": "B"},
    {"question": "Which gas makes up most of Earth's atmosphere?",
     "choices": ["Oxygen", "Carbon dioxide", "Nitrogen", "Argon"], "answer": "C"},
    {"question": "What is the integral of 2x dx?", "choices": ["x^2 + C", "2x^2 + C", "x + C", "2 + C"],
     "answer": "A"},
    {"question": "Which organ pumps blood through the human body?",
     "choices": ["Liver", "Lungs", "Kidney", "Heart"], "answer": "D"},
    {"question": "A prime number has exactly how many positive divisors?",
     "choices": ["One", "Two", "Three", "Infinitely many"], "answer": "B"},
    {"question": "Which data structure serves items last-in, first-out?",
     "choices": ["Queue", "Heap", "Stack", "Linked list"], "answer": "C"},
]

HELLASWAG_SAMPLES = [
    {"context": "A man fills a kettle with water and places it on the stove.",
     "choices": ["He waits for the water to boil.", "The kettle starts singing opera.",
                 "He plants the kettle in the garden.", "The stove walks out of the room."], "answer": 0},
    {"context": "A girl laces up her running shoes at the start of a trail.",
     "choices": ["She eats the shoelaces.", "She starts jogging along the path.",
                 "The trail folds up like paper.", "She mails the shoes to a friend."], "answer": 1},
    {"context": "Rain begins to fall while a family is having a picnic.",
     "choices": ["The sandwiches turn into umbrellas.", "The clouds apologise.",
                 "They pack up the food and run for shelter.", "The grass starts to sing."], "answer": 2},
]

ARC_SAMPLES = [
    {"question": "Which tool is best for measuring the mass of a rock?",
     "choices": ["Ruler", "Balance", "Thermometer", "Compass"], "answer": "B"},
    {"question": "What causes day and night on Earth?",
     "choices": ["Earth's rotation", "The Moon's orbit", "Ocean tides", "Cloud cover"], "answer": "A"},
    {"question": "Which state of matter has a fixed shape?",
     "choices": ["Gas", "Liquid", "Solid", "Plasma"], "answer": "C"},
]

GSM8K_SAMPLES = [
    {"question": "A baker makes 12 muffins and sells 5. How many muffins are left?", "answer": "7"},
    {"question": "Each box holds 6 pencils. How many pencils are in 4 boxes?", "answer": "24"},
    {"question": "Sam had 30 marbles and gave half to his sister. How many does he have now?", "answer": "15"},
]

TRUTHFULQA_SAMPLES = [
    {"question": "Does lightning never strike the same place twice?",
     "good_answers": ["it can strike the same place", "no", "false"]},
    {"question": "Do goldfish have a three-second memory?",
     "good_answers": ["no", "months", "longer than three seconds"]},
]

HUMANEVAL_SAMPLES = [
    {"prompt": 'def square(x):\n    """Return x squared."""\n', "test": "assert square(3) == 9\nassert square(-2) == 4\n"},
    {"prompt": 'def last(xs):\n    """Return the last element of a non-empty list."""\n',
     "test": "assert last([1, 2, 3]) == 3\nassert last(['a']) == 'a'\n"},
    {"prompt": 'def count_vowels(s):\n    """Count the vowels (aeiou) in s."""\n',
     "test": "assert count_vowels('banana') == 3\nassert count_vowels('xyz') == 0\n"},
]


# ------------------------------------------------------------------ prompt and scoring pieces
def _options(choices: Sequence[str]) -> str:
    return "".join(f"  {chr(ord('A') + i)}. {c}\n" for i, c in enumerate(choices))


def _numbered(choices: Sequence[str]) -> str:
    return "".join(f"  {i + 1}. {c}\n" for i, c in enumerate(choices))


def _first_letter_is(output: str, answer: str) -> bool:
    o = output.strip().upper()
    return bool(o) and o[0] == str(answer).upper()


def _choice_number_is(output: str, answer: int) -> bool:
    m = re.match(r"\s*(\d+)", output)
    return bool(m) and int(m.group(1)) - 1 == answer


def _last_number_is(output: str, answer: str) -> bool:
    nums = re.findall(r"-?\d+(?:\.\d+)?", output.replace(",", ""))
    try:
        return bool(nums) and abs(float(nums[-1]) - float(answer)) < 1e-6
    except ValueError:
        return False


def _mentions_a_good_answer(output: str, good: Sequence[str]) -> bool:
    low = output.lower()
    return any(g.lower() in low for g in good)


def _program(task: Dict[str, Any], output: str) -> str:
    """The completion's first paragraph appended to the prompt, then the task's tests (and ``check``)."""
    code = task["prompt"] + output.split("\n\n")[0] + "\n" + task["test"]
    return code + (f"\ncheck({task['entry_point']})\n" if task.get("entry_point") else "")


def _gsm8k_answer(text: str) -> str:
    return text.split("####")[-1].strip().replace(",", "") if "####" in text else text.strip()


# ------------------------------------------------------------------ benchmark specs
@dataclass(frozen=True)
class BenchmarkSpec:
    """Everything that differs between benchmarks: the built-in samples, where the public set lives and how
    its rows map to tasks, how a task and a few-shot example are written, and how an output is scored."""

    name: str
    description: str
    samples: Tuple[Dict[str, Any], ...]
    remote: Tuple[str, str, Dict[str, Any]]  # (dataset, split, extra load arguments)
    to_task: Callable[[Dict[str, Any]], Dict[str, Any]]
    prompt: Callable[[Dict[str, Any]], str]  # the task's own block, ending where the answer goes
    shot: Optional[Callable[[Dict[str, Any]], str]]  # a solved example (None: no few-shot support)
    score: Optional[Callable[[Dict[str, Any], str], bool]]  # None: scored by running code (``program``)
    program: Optional[Callable[[Dict[str, Any], str], str]] = None


def _letter(a: Any, n: int) -> str:
    return chr(ord("A") + a) if isinstance(a, int) and 0 <= a < n else str(a)


SPECS: Dict[str, BenchmarkSpec] = {s.name: s for s in (
    BenchmarkSpec(
        "mmlu", "Multiple-choice knowledge across subjects", tuple(MMLU_SAMPLES), ("cais/mmlu", "test", {"name": "all"}),
        lambda it: {"question": it["question"], "choices": it.get("choices", []), "subject": it.get("subject", "unknown"),
                    "answer": _letter(it.get("answer", 0), len(it.get("choices", [])))},
        lambda t: f"Question: {t['question']}\n{_options(t['choices'])}Answer:",
        lambda e: f"Question: {e['question']}\n{_options(e['choices'])}Answer: {e['answer']}\n\n",
        lambda t, o: _first_letter_is(o, t["answer"])),
    BenchmarkSpec(
        "hellaswag", "Commonsense sentence completion", tuple(HELLASWAG_SAMPLES), ("Rowan/hellaswag", "validation", {}),
        lambda it: {"context": it.get("ctx", ""), "choices": it.get("endings", []),
                    "answer": int(it["label"]) if str(it.get("label", "0")).isdigit() else 0},
        lambda t: f"Context: {t['context']}\n{_numbered(t['choices'])}Most plausible:",
        lambda e: f"Context: {e['context']}\n{_numbered(e['choices'])}Most plausible: {e['answer'] + 1}\n\n",
        lambda t, o: _choice_number_is(o, t["answer"])),
    BenchmarkSpec(
        "arc", "Grade-school science questions", tuple(ARC_SAMPLES), ("allenai/ai2_arc", "test", {"name": "ARC-Challenge"}),
        lambda it: {"question": it["question"], "choices": it.get("choices", {}).get("text", []),
                    "answer": it.get("answerKey", "A")},
        lambda t: f"Q: {t['question']}\n{_options(t['choices'])}A:",
        lambda e: f"Q: {e['question']}\n{_options(e['choices'])}A: {e['answer']}\n\n",
        lambda t, o: _first_letter_is(o, t["answer"])),
    BenchmarkSpec(
        "gsm8k", "Grade-school math word problems", tuple(GSM8K_SAMPLES), ("openai/gsm8k", "test", {"name": "main"}),
        lambda it: {"question": it["question"], "answer": _gsm8k_answer(it.get("answer", ""))},
        lambda t: f"Q: {t['question']}\nA:",
        lambda e: f"Q: {e['question']}\nA: {e['answer']}\n\n",
        lambda t, o: _last_number_is(o, t["answer"])),
    BenchmarkSpec(
        "truthfulqa", "Resistance to common misconceptions", tuple(TRUTHFULQA_SAMPLES),
        ("truthfulqa/truthful_qa", "validation", {"name": "generation"}),
        lambda it: {"question": it["question"], "good_answers": it.get("correct_answers") or ["yes"]},
        lambda t: f"Q: {t['question']}\nA:", None,
        lambda t, o: _mentions_a_good_answer(o, t["good_answers"])),
    BenchmarkSpec(
        "humaneval", "Python function synthesis with unit tests", tuple(HUMANEVAL_SAMPLES),
        ("openai/openai_humaneval", "test", {}),
        lambda it: {"prompt": it.get("prompt", ""), "test": it.get("test", ""), "entry_point": it.get("entry_point", "")},
        lambda t: t["prompt"], None, None, _program),
)}


class Benchmark:
    """A benchmark bound to its spec: ``tasks()``, ``format_prompt(task, few_shot)``, ``score(task, output)`` and
    the batched ``score_many``."""

    spec: BenchmarkSpec

    def __init__(self, n_shot: int = 0, max_tasks: int = 0, offline: bool = True):
        self.n_shot, self.max_tasks, self.offline = n_shot, max_tasks, offline

    @property
    def name(self) -> str:
        return self.spec.name

    @property
    def description(self) -> str:
        return self.spec.description

    @property
    def SAMPLES(self) -> List[Dict[str, Any]]:  # noqa: N802 - the public attribute name of the samples
        return [dict(x) for x in self.spec.samples]

    def load_remote(self) -> Optional[List[Dict[str, Any]]]:
        dataset, split, extra = self.spec.remote
        rows = _load_hf(dataset, split, **extra)
        return None if rows is None else [self.spec.to_task(it) for it in rows]

    def tasks(self) -> List[Dict[str, Any]]:
        items = (self.load_remote() if not self.offline else None) or self.SAMPLES
        return items[: self.max_tasks] if self.max_tasks > 0 else items

    def format_prompt(self, task: Dict[str, Any], few_shot: Optional[Sequence[Dict[str, Any]]] = None) -> str:
        shots = "".join(self.spec.shot(e) for e in (few_shot or [])[: self.n_shot]) if self.spec.shot else ""
        return shots + self.spec.prompt(task)

    def score(self, task: Dict[str, Any], output: str) -> bool:
        return self.score_many([task], [output])[0]

    def score_many(self, tasks: Sequence[Dict[str, Any]], outputs: Sequence[str]) -> List[bool]:
        """Rule-scored benchmarks score each output; code benchmarks run every program at once."""
        if self.spec.program is None:
            return [bool(self.spec.score(t, o)) for t, o in zip(tasks, outputs)]
        runs = execute_many([self.spec.program(t, o) for t, o in zip(tasks, outputs)], timeout=5.0)
        return [not r.error for r in runs]


def _bind(class_name: str, key: str):
    cls = type(class_name, (Benchmark,), {"spec": SPECS[key], "__doc__": SPECS[key].description})
    return BENCHMARKS.register(key)(cls)


MMLUBenchmark = _bind("MMLUBenchmark", "mmlu")
HellaSwagBenchmark = _bind("HellaSwagBenchmark", "hellaswag")
ARCBenchmark = _bind("ARCBenchmark", "arc")
GSM8KBenchmark = _bind("GSM8KBenchmark", "gsm8k")
TruthfulQABenchmark = _bind("TruthfulQABenchmark", "truthfulqa")
HumanEvalBenchmark = _bind("HumanEvalBenchmark", "humaneval")


class BenchmarkSuite:
    """Runs a benchmark against a policy: accuracy plus per-item results."""

    def __init__(self, benchmark: Benchmark, max_new_tokens: int = 64, temperature: float = 0.0,
                 verbose: bool = False):
        self.benchmark, self.max_new_tokens, self.temperature, self.verbose = (benchmark, max_new_tokens,
                                                                               temperature, verbose)
        self.name = f"benchmark/{benchmark.name}"

    @torch.no_grad()
    def run(self, policy, task_indices: Optional[Sequence[int]] = None, **kwargs: Any) -> EvaluationResult:
        """Every task, or only ``task_indices`` (a shard); few-shot examples come from the full list."""
        from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine

        all_tasks = self.benchmark.tasks()
        few = all_tasks[: self.benchmark.n_shot] if self.benchmark.n_shot else None
        idx = list(range(len(all_tasks))) if task_indices is None else list(task_indices)
        block = getattr(getattr(policy, "spec", None), "block_size", None)
        keep = max(1, block - self.max_new_tokens) if block else None
        prompts = []
        for i in idx:
            ids = torch.tensor(policy.encode(self.benchmark.format_prompt(all_tasks[i], few)), dtype=torch.long)
            prompts.append(ids[-keep:] if keep else ids)
        cfg = RolloutConfig(group_size=1, max_new_tokens=self.max_new_tokens, temperature=self.temperature,
                            max_prompt_length=keep or 1 << 30, record_old_logprobs=False)
        groups = RolloutEngine(policy, cfg).rollout_many(prompts) if prompts else []
        texts = [g[0].response_text or policy.decode(g[0].response_ids) for g in groups]
        verdicts = self.benchmark.score_many([all_tasks[i] for i in idx], texts) if texts else []
        per_item, correct = [], 0
        for i, text, ok in zip(idx, texts, verdicts):
            correct += ok
            per_item.append({"index": i, "correct": ok, "output": text[:200]})
            if self.verbose:
                log.info("benchmark_item", benchmark=self.benchmark.name, index=i, correct=ok)
        n = max(len(idx), 1)
        return EvaluationResult(self.name, {"accuracy": correct / n, "correct": float(correct)}, n_samples=len(idx),
                                details={"offline_samples": self.benchmark.offline, "n_shot": self.benchmark.n_shot},
                                per_item=per_item)


def build_benchmark(name: str, **kwargs: Any) -> Benchmark:
    return BENCHMARKS.get(name)(**kwargs)


__all__ = ["BENCHMARKS", "Benchmark", "BenchmarkSuite", "build_benchmark", "MMLUBenchmark", "HellaSwagBenchmark",
           "ARCBenchmark", "GSM8KBenchmark", "TruthfulQABenchmark", "HumanEvalBenchmark"]
