"""Speculative decoding, self-taught reasoning (STaR) and rewards from learned models (CPU only)."""

from __future__ import annotations

import json

import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.core.protocols import Trajectory
from rl_project_b200.models.transformer.model import TransformerLM


def _greedy(model, idx, n):
    """Reference greedy decode: argmax of the full-sequence logits, one token at a time."""
    for _ in range(n):
        nxt = model.full_logits(idx[:, -model.spec.block_size:])[:, -1].argmax(-1, keepdim=True)
        idx = torch.cat([idx, nxt], 1)
    return idx


def _spec(**kw):
    return model_spec_from_preset("tiny", vocab_size=61, block_size=64, **kw)


def test_speculative_greedy_equals_target_greedy_for_any_draft():
    from rl_project_b200.models.generation.speculative import SpeculativeGenerator

    torch.manual_seed(0)
    target, draft = TransformerLM(_spec()).eval(), TransformerLM(_spec()).eval()  # unrelated weights
    prompt = torch.tensor([[3, 14, 15, 9, 2]])
    gen = SpeculativeGenerator(target, draft, k=4)
    out = gen.generate(prompt, max_new_tokens=12, temperature=0.0, top_k=None)
    assert torch.equal(out, _greedy(target, prompt, 12))
    assert 0.0 <= gen.acceptance_rate <= 1.0 and gen.stats["proposed"] > 0


def test_speculative_with_itself_as_draft_accepts_everything():
    from rl_project_b200.models.generation.speculative import SpeculativeGenerator

    torch.manual_seed(1)
    m = TransformerLM(_spec()).eval()
    gen = SpeculativeGenerator(m, m, k=3)
    out = gen.generate(torch.tensor([[1, 2, 3]]), max_new_tokens=20, temperature=1.0, top_k=None)
    assert out.shape[1] >= 3 + 20 and out.shape[1] <= 3 + 20 + 1  # a fully accepted round adds a bonus token
    assert gen.acceptance_rate > 0.95  # p_target == p_draft up to float rounding: ratio 1


def test_speculative_sampling_keeps_the_target_distribution():
    """One speculative step with a mismatched draft: the first emitted token follows the target's
    distribution (Leviathan et al., Theorem 1), checked by frequency over many trials."""
    from rl_project_b200.models.generation.speculative import _accept_or_resample

    torch.manual_seed(2)
    p_t = torch.tensor([[0.5, 0.3, 0.2, 0.0]])
    p_d = torch.tensor([[0.1, 0.1, 0.4, 0.4]])
    counts = torch.zeros(4)
    idx = torch.zeros(1, 0, dtype=torch.long)
    n = 20000
    for _ in range(n):
        tok = torch.multinomial(p_d, 1)
        out, _ = _accept_or_resample(idx, tok, p_t, p_d)
        counts[out[0, -1]] += 1
    assert torch.allclose(counts / n, p_t[0], atol=0.015), counts / n


def test_mtp_self_speculation_greedy_equals_greedy():
    from rl_project_b200.models.generation.speculative import MTPSpeculativeGenerator

    torch.manual_seed(3)
    m = TransformerLM(_spec(n_predict_tokens=3)).eval()
    prompt = torch.tensor([[5, 6, 7, 8]])
    out = MTPSpeculativeGenerator(m).generate(prompt, max_new_tokens=10, temperature=0.0, top_k=None)
    assert torch.equal(out, _greedy(m, prompt, 10))
    with pytest.raises(ValueError):
        MTPSpeculativeGenerator(TransformerLM(_spec()))


def test_star_answer_extraction():
    from rl_project_b200.training.star import answers_match, extract_star_answer, star_prompt

    assert extract_star_answer("so 3 + 4 = 7 <answer> 1,234 </answer> done") == "1234"
    assert extract_star_answer("first 12 then 15") == "15"
    assert extract_star_answer("no digits") is None
    assert answers_match("7.00001", "7") and not answers_match("8", "7") and not answers_match(None, "7")
    assert answers_match("Paris", "paris")
    assert "<answer>NUMBER</answer>" in star_prompt("2+2")


class _ScriptedPolicy:
    """Answers the rows of each generate batch with the scripted texts in turn (a row's single token is the index
    of its text); log-probs come from one parameter."""

    device = torch.device("cpu")
    spec = None

    def __init__(self, texts):
        self.texts, self.calls = list(texts), 0
        self.batches = []
        self.w = torch.nn.Parameter(torch.zeros(()))

    def encode(self, text):
        return [ord(c) % 97 for c in text]

    def decode(self, ids):
        return self.texts[int(ids[0])]

    def generate(self, ids, settings):
        self.batches.append(ids.shape[0])
        rows = [(self.calls + i) % len(self.texts) for i in range(ids.shape[0])]
        self.calls += ids.shape[0]
        return torch.tensor(rows, dtype=torch.long)[:, None]

    def logprobs(self, q, r):
        return torch.full(r.shape, -1.0) + self.w * 0.0 - (self.w - 1.0) ** 2

    def trainable_parameters(self):
        return [self.w]

    def train(self):
        return self

    def eval(self):
        return self

    def state_for_checkpoint(self):
        return {"w": self.w.detach().clone()}


def test_star_keeps_only_correct_rationales(tmp_path):
    from rl_project_b200.data.records import VerifiableTask
    from rl_project_b200.training.star import STaRConfig, STaRTrainer

    tasks = [VerifiableTask(prompt="2+3", answer="5"), VerifiableTask(prompt="4+4", answer="8"),
             VerifiableTask(prompt="1+1", answer="2")]
    pol = _ScriptedPolicy(["2 + 3 = 5 <answer>5</answer>", "it is <answer>9</answer>"])
    tr = STaRTrainer(pol, tasks, STaRConfig(num_rounds=1, samples_per_problem=2, num_problems=2, learning_rate=0.1,
                                            max_new_tokens=8), tmp_path)
    kept = tr.generate_rationales()
    # problem "2+3": one of its two samples is right; problem "4+4": neither says 8
    assert [k["answer"] for k in kept] == ["5"] and "<answer>5</answer>" in kept[0]["rationale"]
    # both problems' prompts have the same length: all four samples came from one batch
    assert pol.batches == [4]
    w0 = float(pol.w)
    loss = tr.sft_on_rationales(kept)
    assert loss == pytest.approx(2.0) and float(pol.w) > w0  # one step on -mean(logprob) = 1 + (w - 1)^2
    res = tr.run()
    assert res["num_rounds"] == 1 and len(res["history"]) == 2
    assert json.loads((tmp_path / "star_results.json").read_text())["method"] == "star"
    with pytest.raises(Exception):
        STaRTrainer(pol, tasks[:1], STaRConfig(), tmp_path)


def test_reward_model_provider_and_blend():
    from rl_project_b200.models.reward import SequenceRewardModel
    from rl_project_b200.rollouts.rewards.learned import BlendedReward, RewardModelProvider

    torch.manual_seed(4)
    spec = _spec()
    rm = SequenceRewardModel(spec)
    prov = RewardModelProvider(rm, max_length=16)
    t = Trajectory(prompt_ids=torch.arange(10), response_ids=torch.arange(10, 22))
    r = prov.score(t).value
    with torch.no_grad():
        ref = float(rm(torch.cat([t.prompt_ids, t.response_ids])[None, -16:]))
    assert r == pytest.approx(ref, rel=1e-5)  # the last max_length tokens are scored
    assert [x.value for x in prov.score_many([t, t])] == pytest.approx([r, r])
    short = Trajectory(prompt_ids=torch.arange(3), response_ids=torch.arange(40, 45))
    alone = prov.score(short).value
    # one right-padded forward for a ragged batch scores every row as if it ran alone
    assert [x.value for x in prov.score_many([t, short])] == pytest.approx([r, alone], rel=1e-4, abs=1e-5)

    blend = BlendedReward(lambda _: 0.5, lambda _: 1.0, neural_weight=0.6)
    res = blend.score(t)
    assert res.value == pytest.approx(0.4 * 0.5 + 0.6 * 1.0) and res.components == {"rule": 0.5, "neural": 1.0}
    assert BlendedReward(lambda _: 0.3).score(t).value == 0.3
    assert BlendedReward(lambda _: 1.0, lambda _: 5.0).score(t).value == 1.0  # clipped to [0, 1]
