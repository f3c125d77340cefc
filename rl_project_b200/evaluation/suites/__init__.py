"""Standard benchmarks with small built-in offline samples.

Each benchmark gives ``tasks()``, ``format_prompt(task, few_shot)`` and
``score(task, output)`` (the interface of
``src/forgeline/evaluation/suites/__init__.py:35-286``).  With ``offline=False``
and the ``datasets`` package present, the public test sets are loaded;
otherwise the built-in samples (written for this project, for wiring and CI,
not for reporting scores) are used.  ``BenchmarkSuite`` decodes every task of
a run in one batched rollout.
"""

from __future__ import annotations

import re
from typing import Any, Dict, List, Optional, Sequence

import torch

from rl_project_b200.core.protocols import EvaluationResult
from rl_project_b200.core.registry import Registry
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.rollouts.tools.python_executor import execute_python

log = get_logger("forgeline.evaluation.suites")

BENCHMARKS: Registry = Registry("benchmark")


def _load_hf(name: str, split: str, **kwargs: Any):
    try:
        from datasets import load_dataset  # optional dependency

        return load_dataset(name, split=split, **kwargs)
    except Exception as exc:  # noqa: BLE001 - offline or not installed
        log.warning("hf_dataset_unavailable", dataset=name, error=str(exc)[:120])
        return None


class Benchmark:
    name = "base"
    description = ""
    SAMPLES: List[Dict[str, Any]] = []

    def __init__(self, n_shot: int = 0, max_tasks: int = 0, offline: bool = True):
        self.n_shot, self.max_tasks, self.offline = n_shot, max_tasks, offline

    def load_remote(self) -> Optional[List[Dict[str, Any]]]:
        return None

    def tasks(self) -> List[Dict[str, Any]]:
        items = (self.load_remote() if not self.offline else None) or list(self.SAMPLES)
        return items[: self.max_tasks] if self.max_tasks > 0 else items

    def format_prompt(self, task: Dict[str, Any], few_shot: Optional[Sequence[Dict[str, Any]]] = None) -> str:
        raise NotImplementedError

    def score(self, task: Dict[str, Any], output: str) -> bool:
        raise NotImplementedError


def _options(choices: Sequence[str]) -> str:
    return "".join(f"  {chr(ord('A') + i)}. {c}\n" for i, c in enumerate(choices))


def _first_letter_is(output: str, answer: str) -> bool:
    o = output.strip().upper()
    return bool(o) and o[0] == str(answer).upper()


@BENCHMARKS.register("mmlu")
class MMLUBenchmark(Benchmark):
    name, description = "mmlu", "Multiple-choice knowledge across subjects"
    SAMPLES = [
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

    def load_remote(self):
        ds = _load_hf("cais/mmlu", "test", name="all")
        if ds is None:
            return None
        out = []
        for it in ds:
            ch, a = it.get("choices", []), it.get("answer", 0)
            out.append({"question": it["question"], "choices": ch, "subject": it.get("subject", "unknown"),
                        "answer": chr(ord("A") + a) if isinstance(a, int) and 0 <= a < len(ch) else str(a)})
        return out

    def format_prompt(self, task, few_shot=None):
        shots = "".join(f"Question: {e['question']}\n{_options(e['choices'])}Answer: {e['answer']}\n\n"
                        for e in (few_shot or [])[: self.n_shot])
        return shots + f"Question: {task['question']}\n{_options(task['choices'])}Answer:"

    def score(self, task, output):
        return _first_letter_is(output, task["answer"])


@BENCHMARKS.register("hellaswag")
class HellaSwagBenchmark(Benchmark):
    name, description = "hellaswag", "Commonsense sentence completion"
    SAMPLES = [
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

    def load_remote(self):
        ds = _load_hf("Rowan/hellaswag", "validation")
        if ds is None:
            return None
        return [{"context": it.get("ctx", ""), "choices": it.get("endings", []),
                 "answer": int(it["label"]) if str(it.get("label", "0")).isdigit() else 0} for it in ds]

    @staticmethod
    def _numbered(choices):
        return "".join(f"  {i + 1}. {c}\n" for i, c in enumerate(choices))

    def format_prompt(self, task, few_shot=None):
        shots = "".join(f"Context: {e['context']}\n{self._numbered(e['choices'])}Most plausible: {e['answer'] + 1}\n\n"
                        for e in (few_shot or [])[: self.n_shot])
        return shots + f"Context: {task['context']}\n{self._numbered(task['choices'])}Most plausible:"

    def score(self, task, output):
        m = re.match(r"\s*(\d+)", output)
        return bool(m) and int(m.group(1)) - 1 == task["answer"]


@BENCHMARKS.register("arc")
class ARCBenchmark(Benchmark):
    name, description = "arc", "Grade-school science questions"
    SAMPLES = [
        {"question": "Which tool is best for measuring the mass of a rock?",
         "choices": ["Ruler", "Balance", "Thermometer", "Compass"], "answer": "B"},
        {"question": "What causes day and night on Earth?",
         "choices": ["Earth's rotation", "The Moon's orbit", "Ocean tides", "Cloud cover"], "answer": "A"},
        {"question": "Which state of matter has a fixed shape?",
         "choices": ["Gas", "Liquid", "Solid", "Plasma"], "answer": "C"},
    ]

    def load_remote(self):
        ds = _load_hf("allenai/ai2_arc", "test", name="ARC-Challenge")
        if ds is None:
            return None
        return [{"question": it["question"], "choices": it.get("choices", {}).get("text", []),
                 "answer": it.get("answerKey", "A")} for it in ds]

    def format_prompt(self, task, few_shot=None):
        shots = "".join(f"Q: {e['question']}\n{_options(e['choices'])}A: {e['answer']}\n\n"
                        for e in (few_shot or [])[: self.n_shot])
        return shots + f"Q: {task['question']}\n{_options(task['choices'])}A:"

    def score(self, task, output):
        return _first_letter_is(output, task["answer"])


@BENCHMARKS.register("gsm8k")
class GSM8KBenchmark(Benchmark):
    name, description = "gsm8k", "Grade-school math word problems"
    SAMPLES = [
        {"question": "A baker makes 12 muffins and sells 5. How many muffins are left?", "answer": "7"},
        {"question": "Each box holds 6 pencils. How many pencils are in 4 boxes?", "answer": "24"},
        {"question": "Sam had 30 marbles and gave half to his sister. How many does he have now?", "answer": "15"},
    ]

    def load_remote(self):
        ds = _load_hf("openai/gsm8k", "test", name="main")
        if ds is None:
            return None
        out = []
        for it in ds:
            a = it.get("answer", "")
            out.append({"question": it["question"],
                        "answer": a.split("####")[-1].strip().replace(",", "") if "####" in a else a.strip()})
        return out

    def format_prompt(self, task, few_shot=None):
        shots = "".join(f"Q: {e['question']}\nA: {e['answer']}\n\n" for e in (few_shot or [])[: self.n_shot])
        return shots + f"Q: {task['question']}\nA:"

    def score(self, task, output):
        nums = re.findall(r"-?\d+(?:\.\d+)?", output.replace(",", ""))
        if not nums:
            return False
        try:
            return abs(float(nums[-1]) - float(task["answer"])) < 1e-6
        except ValueError:
            return False


@BENCHMARKS.register("truthfulqa")
class TruthfulQABenchmark(Benchmark):
    name, description = "truthfulqa", "Resistance to common misconceptions"
    SAMPLES = [
        {"question": "Does lightning never strike the same place twice?",
         "good_answers": ["it can strike the same place", "no", "false"]},
        {"question": "Do goldfish have a three-second memory?",
         "good_answers": ["no", "months", "longer than three seconds"]},
    ]

    def load_remote(self):
        ds = _load_hf("truthfulqa/truthful_qa", "validation", name="generation")
        if ds is None:
            return None
        return [{"question": it["question"], "good_answers": it.get("correct_answers") or ["yes"]} for it in ds]

    def format_prompt(self, task, few_shot=None):
        return f"Q: {task['question']}\nA:"

    def score(self, task, output):
        low = output.lower()
        return any(g.lower() in low for g in task["good_answers"])


@BENCHMARKS.register("humaneval")
class HumanEvalBenchmark(Benchmark):
    name, description = "humaneval", "Python function synthesis with unit tests"
    SAMPLES = [
        {"prompt": 'def square(x):\n    """Return x squared."""\n', "test": "assert square(3) == 9\nassert square(-2) == 4\n"},
        {"prompt": 'def last(xs):\n    """Return the last element of a non-empty list."""\n',
         "test": "assert last([1, 2, 3]) == 3\nassert last(['a']) == 'a'\n"},
        {"prompt": 'def count_vowels(s):\n    """Count the vowels (aeiou) in s."""\n',
         "test": "assert count_vowels('banana') == 3\nassert count_vowels('xyz') == 0\n"},
    ]

    def load_remote(self):
        ds = _load_hf("openai/openai_humaneval", "test")
        if ds is None:
            return None
        return [{"prompt": it.get("prompt", ""), "test": it.get("test", ""), "entry_point": it.get("entry_point", "")}
                for it in ds]

    def format_prompt(self, task, few_shot=None):
        return task["prompt"]

    def score(self, task, output):
        body = output.split("\n\n")[0]
        code = task["prompt"] + body + "\n" + task["test"]
        if task.get("entry_point"):
            code += f"\ncheck({task['entry_point']})\n"
        return not execute_python(code, timeout=5.0).error


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
        per_item, correct = [], 0
        for i, g in zip(idx, groups):
            text = g[0].response_text or policy.decode(g[0].response_ids)
            ok = bool(self.benchmark.score(all_tasks[i], text))
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
