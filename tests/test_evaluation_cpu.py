"""Evaluation suites, benchmarks, inspection, regression rules and results IO (CPU)."""
from __future__ import annotations

import math

import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.core.protocols import EvaluationResult
from rl_project_b200.data.tokenizers import CharTokenizer
from rl_project_b200.evaluation import (BENCHMARKS, BenchmarkSuite, HeldOutLossSuite, PreferenceWinRateSuite,
                                        RecordRewardSuite, RegressionRule, VerifierPassRateSuite, build_benchmark,
                                        evaluate_regression, load_results, measure_engine, measure_generation,
                                        merge_metrics, reward_statistics, save_results)
from rl_project_b200.evaluation.inspection import (activation_flow, attention_patterns, layer_summary,
                                                   weight_statistics)
from rl_project_b200.models.policy import NativePolicy
from rl_project_b200.models.transformer.model import TransformerLM


@pytest.fixture
def policy():
    torch.manual_seed(0)
    tok = CharTokenizer.ascii()
    spec = model_spec_from_preset("tiny", vocab_size=tok.vocab_size, block_size=128)
    return NativePolicy(TransformerLM(spec), tok)


def test_regression_fails_closed():
    rules = [RegressionRule("acc", max_regression=0.01), RegressionRule("loss", "lower_is_better", 0.1, relative=True)]
    ok = evaluate_regression({"acc": 0.5, "loss": 1.05}, {"acc": 0.505, "loss": 1.0}, rules)
    assert ok.passed and not ok.failures()
    bad = evaluate_regression({"acc": 0.4, "loss": float("nan")}, {"acc": 0.5, "loss": 1.0}, rules)
    assert not bad.passed and len(bad.failures()) == 2
    assert not evaluate_regression({"acc": 1.0}, {}, rules[:1]).passed  # baseline missing
    assert not evaluate_regression({}, {}, []).passed  # no rules never passes
    with pytest.raises(ValueError):
        evaluate_regression({}, {}, [RegressionRule("x", direction="sideways")])


def test_results_roundtrip(tmp_path):
    rs = [EvaluationResult("a", {"x": 1.0}, 3, {"k": 1}, [{"i": 0}]), EvaluationResult("b", {"y": 2.0})]
    for name in ("r.json", "r.jsonl"):
        back = load_results(save_results(rs, tmp_path / name))
        assert [r.to_dict() for r in back] == [r.to_dict() for r in rs]
    assert merge_metrics(rs) == {"a/x": 1.0, "b/y": 2.0}


def test_reward_suites():
    s = reward_statistics([0.2, 0.8, 1.0], baseline=0.5)
    assert math.isclose(s["mean"], 2 / 3) and s["pct_above_0.75"] == pytest.approx(200 / 3)
    assert reward_statistics([])["n"] == 0
    r = RecordRewardSuite([{"v": 1}, {"v": 0}], lambda rec: rec["v"]).run()
    assert r.metrics["mean"] == 0.5 and r.details["policy_dependent"] is False
    pw = PreferenceWinRateSuite([{"prompt": "p", "chosen": "long answer", "rejected": "x"}],
                                lambda p, c: len(c)).run()
    assert pw.metrics["win_rate"] == 1.0


def test_benchmark_scoring_rules():
    assert set(BENCHMARKS.names()) == {"mmlu", "hellaswag", "arc", "gsm8k", "truthfulqa", "humaneval"}
    mmlu = build_benchmark("mmlu", n_shot=1)
    t = mmlu.tasks()[1]
    assert mmlu.score(t, f" {t['answer']}. because") and not mmlu.score(t, " Z")
    assert "Question:" in mmlu.format_prompt(t, mmlu.tasks()[:1])
    g = build_benchmark("gsm8k")
    assert g.score({"answer": "24"}, "4 boxes of 6 is 24") and not g.score({"answer": "24"}, "no idea")
    hs = build_benchmark("hellaswag")
    assert hs.score({"answer": 1}, " 2. she runs") and not hs.score({"answer": 1}, "x")
    he = build_benchmark("humaneval")
    task = he.tasks()[0]
    assert he.score(task, "    return x * x\n") and not he.score(task, "    return x + 1\n")
    assert len(build_benchmark("arc", max_tasks=2).tasks()) == 2


def test_benchmark_and_pass_rate_suites_run(policy):
    res = BenchmarkSuite(build_benchmark("arc"), max_new_tokens=4).run(policy)
    assert 0.0 <= res.metrics["accuracy"] <= 1.0 and res.n_samples == 3 and len(res.per_item) == 3
    shard = BenchmarkSuite(build_benchmark("gsm8k"), max_new_tokens=4).run(policy, task_indices=[2])
    assert shard.per_item[0]["index"] == 2

    from rl_project_b200.data.records import VerifiableTask
    from rl_project_b200.rollouts.rewards import build_reward_provider

    tasks = [VerifiableTask(prompt="2+3=", answer="5"), VerifiableTask(prompt="1+1=", answer="2")]
    reward = build_reward_provider({"type": "verifier", "verifier": "math"})
    pr = VerifierPassRateSuite(tasks, reward, max_new_tokens=4).run(policy)
    assert set(pr.metrics) == {"pass_rate", "reward", "malformed_rate"} and pr.n_samples == 2


def test_heldout_loss(corpus_dir, policy):
    from rl_project_b200.data.pretraining import MemmapCorpus

    corpus = MemmapCorpus(corpus_dir, "val", block_size=32)
    r = HeldOutLossSuite(corpus, batches=2, batch_size=2).run(policy.model)
    assert math.isfinite(r.metrics["loss"]) and r.metrics["perplexity"] > 1


def test_performance_measurements(policy):
    m = measure_generation(policy, torch.tensor([5, 6, 7]), max_new_tokens=4, runs=2)
    assert m["tokens_per_second"] > 0 and m["runs"] == 2
    from rl_project_b200.inference import InferenceEngine, SamplingParams

    eng = InferenceEngine(policy.model, max_batch=4)
    e = measure_engine(eng, [[1, 2, 3], [4, 5], [6]], SamplingParams(max_tokens=3, temperature=0.0))
    assert e["tokens_generated"] == 9 and e["requests"] == 3


def test_inspection(policy):
    model = policy.model
    ws = weight_statistics(model)
    assert ws and all(len(w["histogram"]["counts"]) == 20 for w in ws)
    ls = layer_summary(model.spec)
    assert ls[0]["type"] == "embedding" and ls[-1]["type"] == "output" and len(ls) == model.spec.n_layer + 2
    ids = torch.tensor([[1, 2, 3, 4, 5, 6]])
    flow = activation_flow(model, ids)
    assert [f["name"] for f in flow][:1] == ["embedding"] and flow[-1]["name"] == "final_norm"
    pats = attention_patterns(model, ids, per_head=True)
    w = torch.tensor(pats[0]["weights"])
    assert w.shape == (6, 6) and torch.allclose(w.sum(-1), torch.ones(6), atol=1e-5)
    assert torch.triu(w, 1).abs().max() == 0  # causal
