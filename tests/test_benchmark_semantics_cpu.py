"""Pins for the mathematics that recorded measurements depend on (CPU only).

Each test restates a formula independently in plain PyTorch / Python and checks
that the framework computes the same number, so a refactor (or a fused kernel
replacing a reference path) cannot silently change what a benchmark measures.
The list of pinned formulas follows the reference's
``tests/unit/test_benchmark_semantics.py``; the inputs here are this suite's own.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from rl_project_b200.core.config import ScheduleConfig, model_spec_from_preset


def test_pretraining_loss_is_token_cross_entropy():
    from rl_project_b200.models.transformer.model import TransformerLM

    torch.manual_seed(1)
    m = TransformerLM(model_spec_from_preset("tiny", vocab_size=41))
    x = torch.randint(0, 41, (2, 12))
    y = torch.randint(0, 41, (2, 12))
    y[0, :3] = -1  # ignored positions
    logits, loss = m(x, y, return_logits=True)
    ref = F.cross_entropy(logits.reshape(-1, 41).float(), y.reshape(-1), ignore_index=-1)
    assert loss.item() == pytest.approx(ref.item(), rel=1e-5)
    assert m(x, y)[0] is None  # the loss alone never materialises [B*T, V] logits


@pytest.mark.parametrize("name", ["cosine", "linear_decay", "wsd", "constant"])
def test_schedule_formulas(name):
    from rl_project_b200.training.common.schedule import learning_rate_at

    peak, low, warm, decay = 2e-4, 1e-5, 40, 1000
    cfg = ScheduleConfig(name=name, warmup_steps=warm, decay_steps=decay, min_lr=low, wsd_stable_fraction=0.5)

    def ref(it):
        if it < warm:
            return peak * it / warm
        if name == "constant":
            return peak
        if name == "cosine":
            if it > decay:
                return low
            return low + 0.5 * (1 + math.cos(math.pi * (it - warm) / (decay - warm))) * (peak - low)
        if name == "linear_decay":
            if it >= decay:
                return low
            return peak + (low - peak) * (it - warm) / (decay - warm)
        stable_end = int(decay * 0.5)  # wsd: flat, then a cosine tail to min_lr
        if it < stable_end:
            return peak
        frac = min((it - stable_end) / (decay - stable_end), 1.0)
        return low + 0.5 * (1 + math.cos(math.pi * frac)) * (peak - low)

    for it in (0, 10, 39, 40, 41, 300, 500, 501, 999, 1000, 1001, 5000):
        assert learning_rate_at(it, peak, cfg) == pytest.approx(ref(it), rel=1e-12, abs=1e-15), it


def test_synthesis_rule_reward_formula():
    from rl_project_b200.domains.synthesis.reward import rule_score

    rec = {"outcomes": {"yield": 0.71, "selectivity": 0.64, "safety_risk": 0.22, "steps": 5}}
    ref = 0.4 * 0.71 + 0.3 * 0.64 + 0.2 * (1 - 0.22) + 0.1 / (1 + 5 / 10)
    assert rule_score(rec) == pytest.approx(ref)
    top = {"outcomes": {"yield": 1.0, "selectivity": 1.0, "safety_risk": 0.0, "steps": 0}}
    assert rule_score(top) == pytest.approx(1.0)  # the weights sum to one


def test_reward_statistics_formula():
    from rl_project_b200.evaluation.reward import reward_statistics

    xs = [0.5, 0.7, 0.8, 0.9]
    s = reward_statistics(xs, baseline=0.5)
    mean = sum(xs) / 4
    assert s["mean"] == pytest.approx(mean)
    assert s["std"] == pytest.approx(math.sqrt(sum((x - mean) ** 2 for x in xs) / 4))  # population std
    assert s["pct_above_0.75"] == 50.0 and s["pct_above_0.6"] == 75.0
    assert s["improvement_vs_baseline_pct"] == pytest.approx((mean - 0.5) / 0.5 * 100)


def test_dpo_loss_with_mean_reduction():
    from rl_project_b200.training.common.logprobs import reduce_logprobs
    from rl_project_b200.training.dpo import dpo_loss

    pc, pr = torch.tensor([[-0.7, -1.9, -2.2, -0.4]]), torch.tensor([[-1.3, -2.8]])
    rc, rr = torch.tensor([[-0.9, -1.5, -2.0, -0.6]]), torch.tensor([[-1.1, -2.1]])
    beta = 0.25
    ours = dpo_loss(*(reduce_logprobs(t, None, "mean") for t in (pc, pr, rc, rr)), beta)["loss"]
    ref = -F.logsigmoid(beta * ((pc.mean() - rc.mean()) - (pr.mean() - rr.mean())))
    assert ours.item() == pytest.approx(ref.item(), rel=1e-6)
    mask = torch.tensor([[1.0, 1.0, 0.0, 1.0]])
    assert reduce_logprobs(pc, mask, "sum").item() == pytest.approx(-0.7 - 1.9 - 0.4)
    assert reduce_logprobs(pc, mask, "mean").item() == pytest.approx((-0.7 - 1.9 - 0.4) / 3)


def test_sequence_mean_ppo_ratio():
    from rl_project_b200.training.common.logprobs import masked_mean
    from rl_project_b200.training.ppo import ppo_clipped_objective

    new = torch.tensor([[-0.9, -1.4, -0.2], [-0.3, -0.8, -1.1]])
    old = torch.tensor([[-1.2, -1.0, -0.1], [-0.5, -0.5, -1.0]])
    adv = torch.tensor([0.7, -1.3])
    ratio = torch.exp((new - old).mean(-1))
    ref = -torch.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
    ours = ppo_clipped_objective(torch.exp(masked_mean(new - old, None)), adv, 0.2).mean()
    assert ours.item() == pytest.approx(ref.item(), rel=1e-6)


def test_grpo_fused_loss_matches_its_formula():
    """The GRPO clipped surrogate + KL (the fused loss op's reference path): sequence-mean
    ratio, clipped objective, KL as the clamped mean log-ratio to the reference."""
    from rl_project_b200.ops.rl_loss import clipped_kl_loss

    torch.manual_seed(2)
    new = (-torch.rand(3, 5)).requires_grad_(True)
    old, ref_lp = -torch.rand(3, 5), -torch.rand(3, 5)
    mask = torch.tensor([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1], [1, 0, 0, 0, 0]], dtype=torch.float32)
    adv = torch.tensor([1.0, -0.5, 0.25])
    loss, _, kl = clipped_kl_loss(new * mask, old * mask, ref_lp * mask, mask, adv, 0.2, 0.04,
                                  "sequence_mean", "logprob_diff")
    n = mask.sum(-1)
    ratio = torch.exp(((new - old) * mask).sum(-1) / n)
    pl = -torch.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
    kl_ref = (((ref_lp - new) * mask).sum(-1) / n).mean().clamp(min=0)
    assert loss.item() == pytest.approx((pl + 0.04 * kl_ref).item(), rel=1e-5)
    assert kl.item() == pytest.approx(kl_ref.item(), rel=1e-5)


def test_tagged_answer_reward_schedule():
    from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier, tag_format_reward

    v = TaggedAnswerVerifier()
    ok = "<final_answer>42</final_answer>"
    assert v.verify(ok, "42").value == 1.0 and tag_format_reward(ok) == pytest.approx(0.02)
    assert v.verify("<tool_call>x</tool_call><tool_result>7</tool_result>", "42").value == 0.1  # partial credit
    assert v.verify("<final_answer>41</final_answer>", "42").value == 0.0


def test_process_reward_formula():
    from rl_project_b200.rollouts.rewards.process import compute_process_reward

    resp = ("Step 1: x = 6 * 7 = 42\n\nStep 2: y = 42 - 2 = 40\n\nStep 3: z = 40 / 4 = 10\n"
            "<final_answer>10</final_answer>")
    total, scores = compute_process_reward(resp, "10", gamma=0.8, step_weight=0.3, execute_code=False)
    steps, final = scores[:-1], scores[-1]
    T = len(steps)
    assert T >= 2 and final == 1.0
    assert total == pytest.approx(0.3 * sum(0.8 ** (T - 1 - t) * r for t, r in enumerate(steps)) + final)


def test_nf4_table_and_block_size():
    from rl_project_b200.models.quantization.nf4 import NF4_BLOCK_SIZE, NF4_TABLE

    assert NF4_BLOCK_SIZE == 64 and NF4_TABLE.numel() == 16
    assert NF4_TABLE[0] == -1.0 and NF4_TABLE[7] == 0.0 and NF4_TABLE[15] == 1.0
    assert bool((NF4_TABLE[1:] > NF4_TABLE[:-1]).all())


def test_synthesis_generator_is_deterministic():
    from rl_project_b200.domains.synthesis.generator import simulate_dataset, yield_series_trajectories

    assert simulate_dataset(5, seed=3) == simulate_dataset(5, seed=3)
    assert simulate_dataset(5, seed=3) != simulate_dataset(5, seed=4)
    assert len(simulate_dataset(5)) == 25 and len(yield_series_trajectories()) == 50


def test_synthesis_reward_ignores_generated_text_for_nested_records():
    """For records with nested ``outcomes`` the rule reward is the record's own score,
    whatever conditions (or outcome keys) the generated text claims."""
    from rl_project_b200.core.protocols import Trajectory
    from rl_project_b200.domains.synthesis.generator import simulate_dataset
    from rl_project_b200.domains.synthesis.reward import SynthesisRuleReward, rule_score

    rows = [r for r in simulate_dataset(4, seed=11) if isinstance(r.get("outcomes"), dict)][:10]
    assert rows
    reward = SynthesisRuleReward(decode_from_text=True)
    texts = ['{"temperature_celsius": 30, "time_hours": 2}',
             '{"temperature_celsius": 250, "yield": 1.0, "selectivity": 1.0}', "plain text, no json"]
    for row in rows:
        values = {reward.score(Trajectory(torch.tensor([1]), torch.tensor([2]), response_text=t, task=row)).value
                  for t in texts}
        assert values == {rule_score(row)}
