"""Every post-training algorithm runs through the shared Trainer on CPU and learns what it should."""

import math

import pytest
import torch

from rl_project_b200.core.config import AdapterConfig, model_spec_from_preset
from rl_project_b200.data.preference import PreferenceDataset
from rl_project_b200.data.pretraining import MemmapCorpus
from rl_project_b200.data.records import PreferenceRecord, SFTRecord, VerifiableTask
from rl_project_b200.data.supervised import SupervisedDataset
from rl_project_b200.models.policy import NativePolicy
from rl_project_b200.models.reward import SequenceRewardModel
from rl_project_b200.models.transformer.model import TransformerLM
from rl_project_b200.rollouts.agent import AgentRolloutConfig, AgentRolloutEngine
from rl_project_b200.rollouts.engine import RolloutConfig
from rl_project_b200.rollouts.rewards import ConstantReward, LengthReward, VerifierReward, build_reward_provider
from rl_project_b200.rollouts.verifiers import MathVerifier
from rl_project_b200.training import (DAPOAlgorithm, DAPOConfig, DistillationAlgorithm, DistillConfig, DPOAlgorithm,
                                      DPOConfig, GRPOAlgorithm, GRPOConfig, PPOAlgorithm, PPOConfig, PretrainAlgorithm,
                                      PretrainConfig, RewardModelAlgorithm, RewardModelConfig, RLVRConfig, SFTAlgorithm,
                                      SFTConfig, Trainer, build_rlvr_algorithm)


def ok(summary):
    return summary["final_loss"] is not None and math.isfinite(summary["final_loss"])


def test_pretrain_reduces_val_loss(make_ctx, cspec, corpus_dir):
    alg = PretrainAlgorithm(TransformerLM(cspec), MemmapCorpus(corpus_dir, "train", 64), PretrainConfig(batch_size=8),
                            MemmapCorpus(corpus_dir, "val", 64))
    before = alg.evaluate(0)["val_loss"]
    Trainer(make_ctx("pretrain", max_steps=40, batch_size=8, eval_every=0, save_every=0, lr=3e-3), alg).fit()
    assert alg.evaluate(0)["val_loss"] < before


@pytest.mark.parametrize("method", ["none", "lora", "qlora"])
def test_sft_adapters_keep_base_frozen(make_ctx, cspec, char_tok, method):
    recs = [SFTRecord(f"Q: {i}+1?", f" {i + 1}") for i in range(16)]
    adapter = AdapterConfig(method=method, rank=4) if method != "none" else None
    pol = NativePolicy(TransformerLM(cspec), char_tok, adapter=adapter)
    frozen = {n: p.detach().clone() for n, p in pol.model.named_parameters() if not p.requires_grad}
    assert ok(Trainer(make_ctx("sft"), SFTAlgorithm(pol, SupervisedDataset(recs, char_tok, 32), SFTConfig(batch_size=4))).fit())
    for n, p in pol.model.named_parameters():
        if n in frozen:
            assert torch.equal(frozen[n], p)


@pytest.mark.parametrize("reduction", ["sum", "mean"])
def test_dpo_margin_grows(make_ctx, cspec, char_tok, reduction):
    prefs = [PreferenceRecord(f"Q{i}:", " yes", " no") for i in range(8)]
    alg = DPOAlgorithm(NativePolicy(TransformerLM(cspec), char_tok), PreferenceDataset(prefs, char_tok, 16, 8),
                       DPOConfig(batch_size=4, beta=0.5, logprob_reduction=reduction))
    m0 = alg.evaluate(0)["reward_margin"]
    Trainer(make_ctx("dpo", max_steps=15, eval_every=0, save_every=0, lr=5e-3), alg).fit()
    ev = alg.evaluate(0)
    assert ev["reward_margin"] > m0 and ev["preference_accuracy"] == 1.0


def test_batched_dpo_equals_per_example(cspec, char_tok):
    """Right-padded batched log-probs equal one forward per example."""
    from rl_project_b200.training.dpo import sequence_logprobs

    pol = NativePolicy(TransformerLM(cspec), char_tok)
    pol.eval()
    pairs = [(char_tok.encode("Q1: what"), char_tok.encode(" yes")), (char_tok.encode("Q22:"), char_tok.encode(" no!!"))]
    batched = sequence_logprobs(pol, pairs, "sum")
    single = torch.stack([pol.logprobs(torch.tensor(p)[None], torch.tensor(r)[None]).sum() for p, r in pairs])
    assert torch.allclose(batched, single, atol=1e-5)


def test_reward_model_ranks(make_ctx, cspec, char_tok):
    prefs = [PreferenceRecord(f"Q{i}:", " good good good", " bad") for i in range(8)]
    alg = RewardModelAlgorithm(SequenceRewardModel(cspec), PreferenceDataset(prefs, char_tok, 16, 16),
                               RewardModelConfig(batch_size=4))
    Trainer(make_ctx("reward_model", max_steps=20, eval_every=0, save_every=0, lr=3e-3), alg).fit()
    assert alg.evaluate(0)["accuracy"] == 1.0


@pytest.mark.parametrize("ratio_level,kl_mode,entropy_mode", [("sequence_mean", "monitor", "sampled_logprob"),
                                                              ("token", "penalty", "full"),
                                                              ("sequence_mean", "reward", "sampled_logprob")])
def test_ppo_modes(make_ctx, cspec, char_tok, ratio_level, kl_mode, entropy_mode):
    pol = NativePolicy(TransformerLM(cspec), char_tok, value_head=True)
    prompts = [torch.tensor(char_tok.encode(f"Q{i}:")) for i in range(4)]
    alg = PPOAlgorithm(pol, prompts, LengthReward(6),
                       PPOConfig(prompts_per_step=2, samples_per_prompt=2, ppo_epochs=2, ratio_level=ratio_level,
                                 kl_mode=kl_mode, entropy_mode=entropy_mode), RolloutConfig(max_new_tokens=6))
    assert ok(Trainer(make_ctx("ppo", eval_every=0), alg).fit())
    assert "kl" in alg.loss(alg.collect(0), 0, 1)[1]


def test_ppo_epochs_average_equals_one_evaluation_without_dropout(cspec, char_tok):
    """With no active dropout the ``ppo_epochs`` evaluations at fixed weights are identical, so the loss is
    evaluated once; its value and gradient equal the explicit average of ``ppo_epochs`` evaluations."""
    torch.manual_seed(3)
    pol = NativePolicy(TransformerLM(cspec), char_tok, value_head=True)
    pol.value_head.net[0].p = 0.0  # the value head's dropout off: a deterministic forward
    prompts = [torch.tensor(char_tok.encode(f"Q{i}:")) for i in range(3)]
    alg = PPOAlgorithm(pol, prompts, LengthReward(6), PPOConfig(prompts_per_step=2, samples_per_prompt=2, ppo_epochs=3),
                       RolloutConfig(max_new_tokens=5))
    batch = alg.collect(0)
    params = [p for p in alg.parameters() if p.requires_grad]
    loss, _ = alg.loss(batch, 0, 1)
    g1 = torch.autograd.grad(loss, params, allow_unused=True)
    dev = pol.device
    mask, returns = batch.mask.to(dev), batch.rewards.to(dev)
    from rl_project_b200.training.common.advantages import normalize_advantages

    adv = normalize_advantages(returns - batch.old_values.to(dev)).detach()
    runs = [alg._terms(batch, mask, returns, adv, batch.old_logprobs, batch.ref_logprobs)["loss"] for _ in range(3)]
    ref = sum(runs) / 3
    g3 = torch.autograd.grad(ref, params, allow_unused=True)
    assert abs(float(loss) - float(ref)) < 1e-6
    for a, b in zip(g1, g3):
        if a is not None:
            assert torch.allclose(a, b, atol=1e-6)


@pytest.mark.parametrize("objective,ratio_level", [("clipped", "sequence_mean"), ("clipped", "token"),
                                                   ("reinforce", "sequence_mean")])
def test_grpo_objectives(make_ctx, cspec, char_tok, objective, ratio_level):
    tasks = [{"prompt": f"What is {i}+1?", "answer": str(i + 1)} for i in range(4)]
    prompts = [torch.tensor(char_tok.encode(t["prompt"])) for t in tasks]
    alg = GRPOAlgorithm(NativePolicy(TransformerLM(cspec), char_tok), prompts, VerifierReward(MathVerifier()),
                        GRPOConfig(group_size=3, prompts_per_step=2, objective=objective, ratio_level=ratio_level),
                        RolloutConfig(max_new_tokens=6), tasks=tasks)
    assert ok(Trainer(make_ctx("grpo"), alg).fit())


def test_grpo_reuses_rollout_logprobs(cspec, char_tok):
    """Old log-probs recorded at sampling time equal a fresh old-policy pass (so the second pass is skipped)."""
    pol = NativePolicy(TransformerLM(cspec), char_tok)
    prompts = [torch.tensor(char_tok.encode("Q1:")), torch.tensor(char_tok.encode("Q2:"))]
    alg = GRPOAlgorithm(pol, prompts, LengthReward(4), GRPOConfig(group_size=2, prompts_per_step=2),
                        RolloutConfig(max_new_tokens=5))
    from rl_project_b200.rollouts.engine import stack_group

    for grp in alg.collect(0):
        p, r, m = stack_group(grp.trajectories)
        fresh = pol.logprobs(p, r).float() * m
        assert torch.allclose(grp.old_logprobs, fresh, atol=1e-5)


def test_agent_grpo_with_tools(make_ctx, char_tok):
    spec = model_spec_from_preset("tiny", vocab_size=char_tok.vocab_size, block_size=256)
    alg = GRPOAlgorithm(NativePolicy(TransformerLM(spec), char_tok), [{"prompt": "Compute 12 * 3.", "answer": "36"}],
                        build_reward_provider({"type": "tagged"}), GRPOConfig(group_size=2, prompts_per_step=1, agent=True),
                        agent_rollout=AgentRolloutConfig(max_turns=1, max_new_tokens=6, max_context_tokens=200))
    assert ok(Trainer(make_ctx("grpo", max_steps=1, eval_every=0), alg).fit())


def test_agent_engine_injects_tool_results(char_tok):
    outputs = ['<tool_call>{"name": "python_executor", "args": {"code": "print(12*3)"}}</tool_call>',
               "<final_answer>36</final_answer>"]

    class Scripted:
        device = torch.device("cpu")
        pad_token_id = 0

        def __init__(self):
            self.n = 0
            self.seen = []

        def encode(self, t):
            return char_tok.encode(t)

        def decode(self, ids):
            return outputs[self.n - 1]

        def generate(self, ids, settings):
            self.seen.append(char_tok.decode(ids[0].tolist()))
            self.n += 1
            return torch.zeros(1, 1, dtype=torch.long)

    pol = Scripted()
    segs, blocks, final = AgentRolloutEngine(pol, AgentRolloutConfig(max_context_tokens=100000)).run_episode("Solve")
    assert len(segs) == 2 and "36" in blocks[0] and "<tool_result>" in pol.seen[1] and final.endswith("</final_answer>")


def test_dapo_skips_zero_variance_groups(make_ctx, cspec, char_tok):
    pol = NativePolicy(TransformerLM(cspec), char_tok)
    prompts = [torch.tensor(char_tok.encode("Q:"))]
    alg = DAPOAlgorithm(pol, prompts, ConstantReward(1.0), DAPOConfig(group_size=3, prompts_per_step=2),
                        RolloutConfig(max_new_tokens=4))
    groups = alg.collect(0)
    assert all(g.skipped for g in groups)
    loss, metrics = alg.loss(groups, 0, 1)
    assert loss.item() == 0.0 and metrics["groups_skipped"] == 2.0
    alg2 = DAPOAlgorithm(pol, prompts, LengthReward(2), DAPOConfig(group_size=4, prompts_per_step=2, entropy_coef=0.01),
                         RolloutConfig(max_new_tokens=6, temperature=1.5))
    assert ok(Trainer(make_ctx("dapo"), alg2).fit())


def test_dapo_packed_loss_equals_group_by_group(cspec, char_tok):
    """The packed forward over every trajectory of a micro-batch (prompts of different lengths) gives the
    loss of scoring each group alone with its own [G, P] prompt batch."""
    from rl_project_b200.rollouts.engine import stack_group
    from rl_project_b200.training.dapo import dapo_token_objective

    torch.manual_seed(7)
    pol = NativePolicy(TransformerLM(cspec), char_tok)
    prompts = [torch.tensor(char_tok.encode("Q:")), torch.tensor(char_tok.encode("Longer Q?"))]
    cfg = DAPOConfig(group_size=3, prompts_per_step=2, dynamic_sampling=False, kl_coef=0.1, entropy_coef=0.01)
    alg = DAPOAlgorithm(pol, prompts, LengthReward(3), cfg, RolloutConfig(max_new_tokens=6, temperature=1.3))
    groups = alg.collect(0)
    loss, _ = alg.loss(groups, 0, 1)
    pg = kl = ent = 0.0
    ntok = 0.0
    for g in groups:
        prompt, resp, _ = stack_group(g.trajectories, pol.pad_token_id)
        new, e = pol.logprobs_with_entropy(prompt, resp)
        R = g.mask.shape[1]
        new, e = new[:, :R].float() * g.mask, e[:, :R].float()
        per = dapo_token_objective(torch.exp(new - g.old_logprobs) * g.mask, g.advantages[:, None], 0.2, 0.28)
        pg += float((per * g.mask).sum())
        kl += float(((new - g.ref_logprobs) * g.mask).sum())
        ent += float((e * g.mask).sum())
        ntok += float(g.mask.sum())
    ref = (pg + 0.1 * kl - 0.01 * ent) / ntok
    assert abs(float(loss) - ref) < 1e-4, (float(loss), ref)


def test_rlvr_both_optimizers(make_ctx, cspec, char_tok):
    pol = NativePolicy(TransformerLM(cspec), char_tok)
    tasks = [VerifiableTask(prompt=f"What is {i}+1?", answer=str(i + 1)) for i in range(4)]
    for opt in ("dapo", "grpo"):
        cfg = RLVRConfig(optimizer=opt, require_format=True, dapo=DAPOConfig(group_size=2, prompts_per_step=1),
                         grpo=GRPOConfig(group_size=2, prompts_per_step=1))
        alg = build_rlvr_algorithm(pol, tasks, cfg, RolloutConfig(max_new_tokens=8))
        assert alg.name == "rlvr" and ok(Trainer(make_ctx("rlvr", max_steps=2, run=opt), alg).fit())


def test_distillation_with_features(make_ctx, cspec, corpus_dir):
    student = TransformerLM(model_spec_from_preset("tiny", vocab_size=cspec.vocab_size, block_size=64, n_layer=1))
    alg = DistillationAlgorithm(student, TransformerLM(cspec), MemmapCorpus(corpus_dir, "train", 64),
                                DistillConfig(batch_size=4, feature_weight=0.1))
    assert ok(Trainer(make_ctx("distill", eval_every=0), alg).fit())


def test_agent_batched_logprob_matches_per_segment_forwards(char_tok):
    """One forward over the transcript gives each segment the same log-probs as a forward over its own prefix."""
    from rl_project_b200.core.protocols import Trajectory

    torch.manual_seed(0)
    spec = model_spec_from_preset("tiny", vocab_size=char_tok.vocab_size, block_size=256)
    pol = NativePolicy(TransformerLM(spec), char_tok)
    eng = AgentRolloutEngine(pol, AgentRolloutConfig(max_context_tokens=100000))
    trajs = [Trajectory(prompt_ids=torch.zeros(1, dtype=torch.long), response_ids=torch.zeros(1, dtype=torch.long),
                        prompt_text="Q: 2*3?", response_text="", segments=["<tool_call>x</tool_call>", "ok 6"],
                        tool_results=["\n<tool_result>\n6\n</tool_result>\n"]),
             Trajectory(prompt_ids=torch.zeros(1, dtype=torch.long), response_ids=torch.zeros(1, dtype=torch.long),
                        prompt_text="Q: 1+1, say it", response_text="", segments=["two"], tool_results=[])]
    got = eng.trajectories_logprob(trajs)
    with torch.no_grad():
        for t, g in zip(trajs, got):
            ctx, seg_means = t.prompt_text, []
            for i, seg in enumerate(t.segments):
                q, r = torch.tensor(char_tok.encode(ctx))[None], torch.tensor(char_tok.encode(seg))[None]
                seg_means.append(pol.logprobs(q, r).float().mean())
                ctx += seg + (t.tool_results[i] if i < len(t.tool_results) else "")
            assert abs(float(g) - float(torch.stack(seg_means).mean())) < 1e-4
    assert abs(float(eng.trajectory_logprob(trajs[1])) - float(got[1])) < 1e-5


def test_agent_episodes_advance_in_lockstep_batches(char_tok):
    """Episodes of equal context length share one generate call per turn; a finished episode drops out."""
    class Scripted:
        device = torch.device("cpu")
        pad_token_id = 0

        def __init__(self):
            self.batches = []

        def encode(self, t):
            return char_tok.encode(t)

        def decode(self, ids):
            return ['<tool_call>{"name": "python_executor", "args": {"code": "print(2)"}}</tool_call>',
                    "<final_answer>2</final_answer>"][int(ids[0])]

        def generate(self, ids, settings):
            # turn 1: row 0 calls the tool, row 1 answers; turn 2: the remaining row answers
            self.batches.append(ids.shape[0])
            return torch.tensor([[0], [1]] if ids.shape[0] == 2 else [[1]], dtype=torch.long)

    pol = Scripted()
    out = AgentRolloutEngine(pol, AgentRolloutConfig(max_context_tokens=100000)).run_episodes(["P1", "P2"])
    assert pol.batches == [2, 1]
    (segs0, obs0, final0), (segs1, obs1, final1) = out
    assert len(segs0) == 2 and "2" in obs0[0] and final0.endswith("</final_answer>")
    assert len(segs1) == 1 and obs1 == []


def test_rlvr_pass_rate_scores_one_batched_answer_per_task(cspec, char_tok):
    from rl_project_b200.training.rlvr import RLVRConfig, build_verifiable_reward, evaluate_pass_rate

    pol = NativePolicy(TransformerLM(cspec), char_tok)
    tasks = [VerifiableTask(prompt=f"What is {i}+1?", answer=str(i + 1)) for i in range(5)]
    res = evaluate_pass_rate(pol, tasks, build_verifiable_reward(RLVRConfig(task_type="math")), max_new_tokens=4,
                             limit=3)
    assert res["n"] == 3 and 0.0 <= res["pass_rate"] <= 1.0 and 0.0 <= res["malformed_rate"] <= 1.0
    assert evaluate_pass_rate(pol, [], build_verifiable_reward(RLVRConfig()))["n"] == 0


def test_distillation_loss_value_and_gradient_match_autograd(monkeypatch):
    """The chunked op with its analytic gradient equals the plain autograd formula (several row chunks)."""
    import torch.nn.functional as F

    from rl_project_b200.training import distill

    monkeypatch.setattr(distill, "_CHUNK_ELEMS", 3 * 50)  # 3 rows per chunk
    torch.manual_seed(0)
    s = torch.randn(2, 5, 50, dtype=torch.float64, requires_grad=True)
    t = torch.randn(2, 5, 50, dtype=torch.float64)
    y = torch.randint(0, 50, (2, 5))
    y[0, :2] = -1
    T, a = 3.0, 0.6
    got = distill.distillation_loss(s, t, y, T, a)
    (g_got,) = torch.autograd.grad(2.0 * got, s)
    s2 = s.detach().clone().requires_grad_(True)
    kl = F.kl_div(F.log_softmax(s2.reshape(-1, 50) / T, -1), F.softmax(t.reshape(-1, 50) / T, -1),
                  reduction="batchmean") * T ** 2
    ref = a * kl + (1 - a) * F.cross_entropy(s2.reshape(-1, 50), y.reshape(-1), ignore_index=-1)
    (g_ref,) = torch.autograd.grad(2.0 * ref, s2)
    # the op works in fp32 whatever the input dtype
    assert abs(float(got) - float(ref)) < 1e-5 * abs(float(ref))
    assert torch.allclose(g_got, g_ref, atol=1e-7)


def test_rlaif_trainer_round_with_batched_generation_and_packed_dpo(cspec, char_tok, tmp_path):
    """One RLAIF round: K candidates per task from one batched generation, judged (a content-hash judge and
    the policy's own judge), pairs past the score gap, one reference-free DPO step over all pairs."""
    from rl_project_b200.training.rlaif import RLAIFConfig, RLAIFTrainer

    torch.manual_seed(11)
    pol = NativePolicy(TransformerLM(cspec), char_tok)
    tasks = [VerifiableTask(prompt=f"What is {i}+2?", answer=str(i + 2)) for i in range(2)]
    cfg = RLAIFConfig(num_rounds=1, candidates_per_prompt=3, pair_gap=0.5, max_new_tokens=8, temperature=1.5,
                      judge_max_tokens=4, num_problems=2)
    w0 = [p.detach().clone() for p in pol.trainable_parameters()]
    res = RLAIFTrainer(pol, tasks, cfg, tmp_path, judge_fn=lambda q, r: (sum(map(ord, r)) % 11) / 10.0).run()
    h = res["history"][0]
    assert h["pairs"] > 0 and math.isfinite(h["dpo_loss"])
    assert any(not torch.equal(a, b) for a, b in zip(w0, pol.trainable_parameters()))
    # the policy as its own judge: scores parsed from its replies (fallback 0.5 for unparsable text)
    own = RLAIFTrainer(pol, tasks, cfg, tmp_path / "own")
    scores = own._judge_many([("1+1?", "2"), ("2+2?", "4")])
    assert len(scores) == 2 and all(0.0 <= s <= 1.0 for s in scores)
