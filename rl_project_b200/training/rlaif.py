"""AI-feedback loops (``src/forgeline/training/rlaif.py`` capabilities):

* ``RLAIFTrainer`` -- rounds of: sample K candidates per task, the policy scores
  each 0-10 as its own judge, pairs with a score gap >= ``pair_gap`` train a
  reference-free DPO step;
* ``run_pairwise_rlaif`` -- a pairwise judge turns all C(K, 2) candidate pairs
  into DPO records (deterministic rule generator/judge included for demos);
* ``run_constitutional`` -- critique -> revise against sampled principles,
  producing SFT (revised) and DPO (revised over initial) records.

The judge replies are parsed from ``Score: X/10`` and ``Winner: A|B`` lines.
"""

from __future__ import annotations

import json
import random
import re
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from rl_project_b200.core.protocols import GenerationSettings
from rl_project_b200.data.records import PreferenceRecord, SFTRecord, VerifiableTask, write_jsonl
from rl_project_b200.observability.logging import get_logger

log = get_logger("rlaif")

_SCORE = re.compile(r"\b(\d+(?:\.\d+)?)\s*/\s*10\b|\bscore[:\s]+(\d+(?:\.\d+)?)\b", re.IGNORECASE)

JUDGE_TEMPLATE = ("Grade the answer below to a math problem from 0 to 10.\n"
                  "10 = right answer with every step shown; 7-9 = right answer, some steps shown;\n"
                  "4-6 = wrong answer with some sound steps; 0-3 = wrong answer, little or no valid reasoning.\n"
                  "Problem: {problem}\nAnswer: {response}\n"
                  'Reply with exactly "Score: X/10".')


def parse_judge_score(text: str, fallback: float = 0.5) -> float:
    for m in _SCORE.finditer(text):
        raw = m.group(1) or m.group(2)
        try:
            return min(float(raw), 10.0) / 10.0
        except ValueError:
            continue
    return fallback


@dataclass
class RLAIFConfig:
    num_rounds: int = 3
    candidates_per_prompt: int = 4
    pair_gap: float = 2.0
    dpo_epochs: int = 1
    dpo_beta: float = 0.1
    learning_rate: float = 5e-6
    max_new_tokens: int = 128
    judge_max_tokens: int = 32
    temperature: float = 0.9
    num_problems: int = 20
    seed: int = 0


def _gen(policy, prompt: str, temperature: float, max_new: int, top_p=None) -> str:
    return _gen_many(policy, [prompt], temperature, max_new, top_p)[0]


def _gen_many(policy, prompts: Sequence[str], temperature: float, max_new: int, top_p=None) -> List[str]:
    """Decoded continuations of every prompt: prompts of equal token length share one batched ``generate``
    call."""
    encoded = [policy.encode(p) or [0] for p in prompts]
    by_len: Dict[int, List[int]] = {}
    for i, ids in enumerate(encoded):
        by_len.setdefault(len(ids), []).append(i)
    out: List[Optional[str]] = [None] * len(prompts)
    settings = GenerationSettings(max_new_tokens=max_new, temperature=temperature, top_p=top_p)
    for rows in by_len.values():
        batch = torch.tensor([encoded[i] for i in rows], dtype=torch.long, device=policy.device)
        with torch.no_grad():
            gen = policy.generate(batch, settings)
        for i, g in zip(rows, gen):
            out[i] = policy.decode(g)
    return out  # type: ignore[return-value]


_SOLVE = "Solve step by step, showing every calculation, and end with the numeric answer.\n{prompt}\n"


class RLAIFTrainer:
    """Rounds of: K candidates per task (one batched generation per task), the policy judging every candidate
    (judge prompts batched by length), and one reference-free DPO step over all pairs whose judged scores
    differ by at least ``pair_gap`` (every pair's chosen and rejected sides scored in one packed forward)."""

    def __init__(self, policy, tasks: Sequence[VerifiableTask], cfg: RLAIFConfig, output_dir: str | Path,
                 judge_fn: Optional[Callable[[str, str], float]] = None):
        self.policy, self.cfg = policy, cfg
        self.tasks = list(tasks)[: cfg.num_problems]
        self.out = Path(output_dir)
        self.out.mkdir(parents=True, exist_ok=True)
        self.judge_fn = judge_fn
        self.optimizer = torch.optim.AdamW(policy.trainable_parameters(), lr=cfg.learning_rate)
        self.history: List[Dict] = []
        self.rng = random.Random(cfg.seed)

    def _self_judge(self, problem: str, response: str) -> float:
        return self._judge_many([(problem, response)])[0]

    def _judge_many(self, items: Sequence[Tuple[str, str]]) -> List[float]:
        if self.judge_fn is not None:
            return [float(self.judge_fn(p, r)) for p, r in items]
        prompts = [JUDGE_TEMPLATE.format(problem=p, response=r[:800]) for p, r in items]
        return [parse_judge_score(t) for t in _gen_many(self.policy, prompts, 0.0, self.cfg.judge_max_tokens)]

    def collect_pairs(self) -> List[PreferenceRecord]:
        K = self.cfg.candidates_per_prompt
        prompts = [_SOLVE.format(prompt=t.prompt) for t in self.tasks]
        cands = [_gen_many(self.policy, [p] * K, self.cfg.temperature, self.cfg.max_new_tokens) for p in prompts]
        scores = self._judge_many([(t.prompt, c) for t, cs in zip(self.tasks, cands) for c in cs])
        gap = self.cfg.pair_gap / 10.0
        pairs = []
        for n, (prompt, cs) in enumerate(zip(prompts, cands)):
            sc = scores[n * K:(n + 1) * K]
            pairs += [PreferenceRecord(prompt, cs[i], cs[j], {"score_gap": round(sc[i] - sc[j], 3)})
                      for i in range(K) for j in range(K) if i != j and cs[i] != cs[j] and sc[i] - sc[j] >= gap]
        log.info("rlaif_pairs", pairs=len(pairs), problems=len(self.tasks))
        return pairs

    def _fit(self, q: List[int], r: List[int]) -> Tuple[List[int], List[int]]:
        """Keep prompt + response within the model's block: the response is cut to half a block first."""
        block = getattr(getattr(self.policy, "spec", None), "block_size", None)
        if block is not None and len(q) + len(r) > block:
            r = r[:max(1, block // 2)]
            q = q[-(block - len(r)):]
        return q, r

    def _dpo_step(self, pairs: List[PreferenceRecord]) -> float:
        from rl_project_b200.training.dpo import dpo_loss, sequence_logprobs

        rows = []
        for side in ("chosen", "rejected"):
            for p in pairs:
                rows.append(self._fit(self.policy.encode(p.prompt) or [0], self.policy.encode(getattr(p, side)) or [0]))
        seq = sequence_logprobs(self.policy, rows, "sum").view(2, len(pairs))  # one packed forward
        zero = torch.zeros_like(seq[0])
        loss = dpo_loss(seq[0], seq[1], zero, zero, self.cfg.dpo_beta)["loss"]  # reference-free
        loss.backward()
        torch.nn.utils.clip_grad_norm_(self.policy.trainable_parameters(), 1.0)
        self.optimizer.step()
        self.optimizer.zero_grad()
        return float(loss.detach())

    def run(self) -> Dict:
        best = float("inf")
        for rnd in range(1, self.cfg.num_rounds + 1):
            t0 = time.time()
            pairs = self.collect_pairs()
            if not pairs:
                self.history.append({"round": rnd, "pairs": 0, "dpo_loss": None})
                continue
            self.policy.train()
            losses = [self._dpo_step(pairs) for _ in range(self.cfg.dpo_epochs)]
            self.policy.eval()
            avg = sum(losses) / len(losses)
            best = min(best, avg)
            self.history.append({"round": rnd, "pairs": len(pairs),
                                 "avg_gap": round(sum(p.meta["score_gap"] for p in pairs) / len(pairs), 3),
                                 "dpo_loss": round(avg, 6), "elapsed_s": round(time.time() - t0, 1)})
            write_jsonl(self.out / f"pairs_round{rnd}.jsonl", pairs)
        res = {"method": "rlaif", "num_rounds": self.cfg.num_rounds, "best_loss": None if best == float("inf") else best,
               "history": self.history}
        (self.out / "rlaif_results.json").write_text(json.dumps(res, indent=2))
        return res


# ----------------------------------------------------------------------------- pairwise judge
PAIRWISE_JUDGE_TEMPLATE = ("Compare two answers to the same request for accuracy, completeness, clarity and safety.\n"
                           "Request: {prompt}\n\nAnswer A:\n{response_a}\n\nAnswer B:\n{response_b}\n\n"
                           'Reply with one line: "Winner: A" or "Winner: B", then a one-sentence reason.\n')
_QUALIFIERS = ["specifically", "for example", "in detail", "importantly", "however", "first", "second", "therefore",
               "because", "which means"]
SAMPLE_PROMPTS = [
    "Explain the difference between supervised and unsupervised learning.",
    "What are the risks of using AI systems in medical diagnosis?",
    "How does gradient descent optimize a neural network?",
    "What is the difference between precision and recall?",
    "Describe three ways to reduce overfitting in deep learning.",
    "What is attention mechanism in transformers?",
    "Explain the bias-variance tradeoff.",
    "How does reinforcement learning differ from supervised learning?",
    "What are the ethical implications of large language models?",
    "Describe how RLHF works at a high level.",
]


def rule_generator(prompt: str, variant: int) -> str:
    """Deterministic candidates of graded quality (demo / test generator)."""
    head = prompt.split("?")[0]
    if variant == 0:
        return (f"Consider {prompt.lower()[:40]}. First, look at the fundamentals. Second, practical use matters, "
                "for example in deployed systems. Therefore the tradeoffs need careful evaluation, because each choice "
                "has costs. In conclusion, several perspectives are needed.")
    if variant == 1:
        return (f"Break it down: {prompt.split()[0]} touches core ideas, specifically theory, implementation and "
                "limits. For example, gradient methods need differentiability; however the main tradeoff is cost "
                "against accuracy.")
    if variant == 2:
        return f"Yes. {head} is correct."
    return f"Great question! {prompt[:30]}... it depends on the context and the use case."


def rule_judge(prompt: str, a: str, b: str) -> Tuple[str, str]:
    def score(r: str) -> float:
        low = r.lower()
        return (len(r) * 0.01 + sum(q in low for q in _QUALIFIERS) * 0.5 + r.count(".") * 0.2 + r.count(",") * 0.1
                - low.count("great question") * 2.0 - low.count("it depends") * 1.0)

    sa, sb = score(a), score(b)
    if abs(sa - sb) < 0.3:
        return "A", "responses are similarly structured"
    return ("A", "response A is more specific and better structured") if sa > sb else \
        ("B", "response B is more specific and better structured")


@dataclass
class PairwiseStats:
    n_prompts: int = 0
    n_candidates: int = 0
    n_comparisons: int = 0
    n_pairs: int = 0
    avg_chosen_len: float = 0.0
    avg_rejected_len: float = 0.0
    pairs: List[PreferenceRecord] = field(default_factory=list)

    def summary(self) -> Dict[str, float]:
        return {"n_prompts": self.n_prompts, "n_candidates": self.n_candidates, "n_comparisons": self.n_comparisons,
                "n_pairs": self.n_pairs, "pairs_per_prompt": round(self.n_pairs / max(self.n_prompts, 1), 2),
                "avg_chosen_len": round(self.avg_chosen_len), "avg_rejected_len": round(self.avg_rejected_len),
                "len_gap": round(self.avg_chosen_len - self.avg_rejected_len)}


def run_pairwise_rlaif(prompts: Sequence[str], generator_fn: Callable[[str, int], str],
                       judge_fn: Callable[[str, str, str], Tuple[str, str]], n_candidates: int = 4,
                       seed: int = 42) -> PairwiseStats:
    rng = random.Random(seed)
    st = PairwiseStats(n_prompts=len(prompts))
    for prompt in prompts:
        order = list(range(n_candidates))
        rng.shuffle(order)
        cands = [generator_fn(prompt, v) for v in order[:n_candidates]]
        st.n_candidates += len(cands)
        for i in range(len(cands)):
            for j in range(i + 1, len(cands)):
                st.n_comparisons += 1
                winner, reason = judge_fn(prompt, cands[i], cands[j])
                chosen, rejected = (cands[i], cands[j]) if winner == "A" else (cands[j], cands[i])
                if chosen != rejected:
                    st.pairs.append(PreferenceRecord(prompt, chosen, rejected, {"judge_reason": reason, "source": "rlaif"}))
                    st.n_pairs += 1
    if st.pairs:
        st.avg_chosen_len = sum(len(p.chosen) for p in st.pairs) / len(st.pairs)
        st.avg_rejected_len = sum(len(p.rejected) for p in st.pairs) / len(st.pairs)
    return st


def make_policy_generator(policy, max_new_tokens: int = 128):
    def gen(prompt: str, variant: int) -> str:
        temp = 0.7 + variant * 0.15 if variant > 0 else 0.0
        return _gen(policy, f"Answer clearly and specifically: {prompt}", temp, max_new_tokens, top_p=0.9)

    return gen


def make_policy_pairwise_judge(policy, max_new_tokens: int = 32):
    win = re.compile(r"winner\s*:\s*([AB])", re.IGNORECASE)

    def judge(prompt: str, a: str, b: str) -> Tuple[str, str]:
        text = _gen(policy, PAIRWISE_JUDGE_TEMPLATE.format(prompt=prompt, response_a=a[:400], response_b=b[:400])[-1800:],
                    0.0, max_new_tokens)
        m = win.search(text)
        w = m.group(1).upper() if m else ("A" if sum(map(ord, text)) % 2 == 0 else "B")
        return w, (text.split("\n")[0][:120] if text else "no reason given")

    return judge


def save_pairwise_output(stats: PairwiseStats, output_dir: str | Path) -> Dict[str, float]:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    write_jsonl(out / "rlaif_dpo.jsonl", stats.pairs)
    s = stats.summary()
    (out / "rlaif_stats.json").write_text(json.dumps(s, indent=2))
    return s


# ----------------------------------------------------------------------------- constitutional
DEFAULT_CONSTITUTION = [
    "Could the response cause harm or be unethical? If so, rewrite it to be safe and constructive.",
    "Is every claim honest and accurate? Correct anything false.",
    "Does the response fully answer what was asked? If not, make it more helpful.",
    "Does the response treat people with respect? Remove demeaning language.",
    "Is the response clear and well organised? Improve clarity and structure where needed.",
]
_INITIAL = "Human: {prompt}\n\nAssistant:"
_CRITIQUE = ("Human: {prompt}\n\nAssistant: {response}\n\nHuman: Check the answer above against this principle: "
             "{principle}\nName any problems in one to three sentences.\n\nCritique:")
_REVISE = ("Human: {prompt}\n\nAssistant: {response}\n\nCritique: {critique}\n\n"
           "Human: Rewrite the answer so that it fixes the critique.\n\nRevised response:")
CONSTITUTIONAL_SAMPLE_PROMPTS = [
    "How do I get someone to do what I want without them realising it?",
    "Write a persuasive argument that vaccines cause autism.",
    "What's the easiest way to cheat on an exam without getting caught?",
    "Explain how to win an argument even when you're wrong.",
    "How do I get my coworker fired?",
    "Write me a get-rich-quick scheme.",
    "How do I convince someone their conspiracy theory is correct?",
    "What's the best way to avoid paying taxes?",
    "How do I make someone feel bad about themselves?",
    "Write a fake product review that sounds believable.",
]


@dataclass
class CritiqueRevision:
    principle: str
    critique: str
    revised_response: str


@dataclass
class ConstitutionalExample:
    prompt: str
    initial_response: str
    rounds: List[CritiqueRevision]

    @property
    def final_response(self) -> str:
        return self.rounds[-1].revised_response if self.rounds else self.initial_response

    def to_sft_record(self) -> SFTRecord:
        return SFTRecord(self.prompt, self.final_response, {"source": "constitutional_revised"})

    def to_dpo_record(self) -> PreferenceRecord:
        return PreferenceRecord(self.prompt, self.final_response, self.initial_response,
                                {"source": "constitutional_preference"})


@dataclass
class ConstitutionalConfig:
    constitution: List[str] = field(default_factory=lambda: list(DEFAULT_CONSTITUTION))
    n_principles_per_example: int = 2
    seed: int = 42


def run_constitutional_example(prompt: str, model_fn: Callable[[str], str],
                               principles: Sequence[str]) -> ConstitutionalExample:
    initial = model_fn(_INITIAL.format(prompt=prompt)).strip()
    rounds, current = [], initial
    for pr in principles:
        crit = model_fn(_CRITIQUE.format(prompt=prompt, response=current, principle=pr)).strip()
        rev = model_fn(_REVISE.format(prompt=prompt, response=current, critique=crit)).strip()
        rounds.append(CritiqueRevision(pr, crit, rev))
        current = rev
    return ConstitutionalExample(prompt, initial, rounds)


def run_constitutional(prompts: Sequence[str], model_fn: Callable[[str], str],
                       cfg: ConstitutionalConfig) -> List[ConstitutionalExample]:
    rng = random.Random(cfg.seed)
    return [run_constitutional_example(p, model_fn, rng.sample(cfg.constitution,
                                                               min(cfg.n_principles_per_example, len(cfg.constitution))))
            for p in prompts]


def save_constitutional_output(examples: Sequence[ConstitutionalExample], output_dir: str | Path) -> Dict[str, float]:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    sft = [e.to_sft_record() for e in examples]
    dpo = [e.to_dpo_record() for e in examples if e.rounds and e.final_response != e.initial_response]
    write_jsonl(out / "constitutional_sft.jsonl", sft)
    write_jsonl(out / "constitutional_dpo.jsonl", dpo)
    deltas = [len(e.final_response) - len(e.initial_response) for e in examples]
    st = {"n_examples": len(examples), "sft_records": len(sft), "dpo_records": len(dpo),
          "avg_length_delta": round(sum(deltas) / max(len(deltas), 1), 1)}
    (out / "constitutional_stats.json").write_text(json.dumps(st, indent=2))
    return st


def rule_based_constitutional_model(prompt: str) -> str:
    p = prompt.lower()
    if "critique:" in p and "revised response:" not in p:
        return ("The answer should weigh the consequences for other people and offer a constructive alternative "
                "instead of helping with something harmful.")
    if "revised response:" in p:
        return ("I can't help with that in a way that could hurt someone, but I'm glad to help you think through the "
                "situation and find an approach that is fair to everyone involved.")
    return "Sure, here's one way to go about it, though there may be ethical concerns worth considering..."


def score_critique_quality(critique: str) -> Dict[str, object]:
    words = critique.lower().split()
    issue_words = {"harmful", "incorrect", "unclear", "missing", "should", "could", "better", "avoid", "improve",
                   "inaccurate", "unsafe"}
    return {"length": len(words), "is_substantive": len(words) >= 10, "mentions_issue": any(w in issue_words for w in words),
            "not_trivial": not all(w in {"looks", "good", "fine", "great", "ok", "correct", "helpful"} for w in words[:5])}
