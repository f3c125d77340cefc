"""Training utilities, verifiers, rewards and tools (the reference's unit/test_training_utils.py and
unit/test_rollouts_rewards.py are the model)."""
import math

import pytest
import torch

from rl_project_b200.core.config import OptimizerConfig, ScheduleConfig
from rl_project_b200.core.errors import InvalidRewardError
from rl_project_b200.core.protocols import RewardResult, Trajectory


# ------------------------------------------------------------------ schedules / optimizer / advantages
def test_schedules():
    from rl_project_b200.training.common.schedule import learning_rate_at

    cos = ScheduleConfig(name="cosine", warmup_steps=10, decay_steps=110, min_lr=0.1)
    assert learning_rate_at(0, 1.0, cos) == 0.0 and learning_rate_at(5, 1.0, cos) == 0.5
    assert learning_rate_at(10, 1.0, cos) == pytest.approx(1.0)
    assert learning_rate_at(60, 1.0, cos) == pytest.approx(0.55)  # half way down the cosine
    assert learning_rate_at(500, 1.0, cos) == 0.1
    wsd = ScheduleConfig(name="wsd", warmup_steps=0, decay_steps=100, min_lr=0.0, wsd_stable_fraction=0.8)
    assert learning_rate_at(79, 2.0, wsd) == 2.0 and learning_rate_at(100, 2.0, wsd) == pytest.approx(0.0)
    lin = ScheduleConfig(name="linear_decay", warmup_steps=0, decay_steps=100, min_lr=0.0)
    assert learning_rate_at(50, 1.0, lin) == pytest.approx(0.5)
    assert learning_rate_at(7, 3e-4, ScheduleConfig(name="constant", warmup_steps=0)) == 3e-4


def test_optimizer_groups_decay_only_matrices():
    from rl_project_b200.training.common.optim import build_optimizer, param_groups

    lin = torch.nn.Linear(4, 3)
    groups = param_groups(list(lin.parameters()), OptimizerConfig(weight_decay=0.1))
    assert [len(g["params"]) for g in groups] == [1, 1] and [g["weight_decay"] for g in groups] == [0.1, 0.0]
    opt = build_optimizer(lin.parameters(), OptimizerConfig(name="adam"), torch.device("cpu"))
    assert isinstance(opt, torch.optim.Adam)


def test_gae_and_group_advantages():
    from rl_project_b200.training.common.advantages import compute_gae, group_relative_advantages, grouped_advantages

    r, v = torch.tensor([1.0, 0.0, 2.0]), torch.tensor([0.5, 0.5, 0.5, 0.0])
    adv, ret = compute_gae(r, v, gamma=0.9, lam=0.8)
    d2 = 2.0 + 0.9 * 0.0 - 0.5
    d1 = 0.0 + 0.9 * 0.5 - 0.5
    d0 = 1.0 + 0.9 * 0.5 - 0.5
    want = [d0 + 0.72 * (d1 + 0.72 * d2), d1 + 0.72 * d2, d2]
    assert adv.tolist() == pytest.approx(want) and ret.tolist() == pytest.approx([a + 0.5 for a in want])
    rewards = torch.tensor([1.0, 0.0, 0.0, 1.0, 5.0, 5.0, 5.0, 5.0])
    g = grouped_advantages(rewards, 4)
    assert g[:4].tolist() == pytest.approx(group_relative_advantages(rewards[:4]).tolist())
    assert g[4:].abs().max() < 1e-6  # zero-variance group: no signal
    assert group_relative_advantages(torch.tensor([3.0])).item() == 0.0


def test_logprob_reductions_and_kl():
    from rl_project_b200.training.common.logprobs import kl_k3, kl_logprob_diff, masked_mean, reduce_logprobs

    lp = torch.tensor([[-1.0, -2.0, -3.0], [-1.0, -1.0, 0.0]])
    m = torch.tensor([[1.0, 1.0, 0.0], [1.0, 0.0, 0.0]])
    assert reduce_logprobs(lp, m, "sum").tolist() == [-3.0, -1.0]
    assert reduce_logprobs(lp, m, "mean").tolist() == [-1.5, -1.0]
    ref = lp + 0.1
    assert kl_logprob_diff(ref, lp, m).tolist() == pytest.approx([0.1, 0.1])
    d = torch.tensor(0.1)
    assert kl_k3(ref, lp, m).tolist() == pytest.approx([float(d.exp() - d - 1)] * 2)
    assert masked_mean(lp, torch.zeros_like(m)).tolist() == [0.0, 0.0]  # empty masks do not divide by zero


# ------------------------------------------------------------------ verifiers / rewards / tools
def test_math_verifier_answers_and_partial_credit():
    from rl_project_b200.rollouts.verifiers import MathVerifier

    v = MathVerifier()
    assert v.verify("so the result is \\boxed{42}", "42").value == 1.0
    assert v.verify("#### 1,000", "1000").passed
    assert v.verify("#### 3.14159", "3.1416").value == 0.5  # not exact, within 1 % relative: partial credit
    # "the answer is" captures up to the first period (the reference's pattern): 3.14159 reads as 3
    assert v.extract_answer("The answer is 3.14159") == "3"
    assert v.verify("nothing numeric here", "7").value == 0.0


def test_tagged_exact_format_and_parity():
    from rl_project_b200.rollouts.verifiers import (ExactMatchVerifier, FormatVerifier, LastTokenParityVerifier,
                                                    TaggedAnswerVerifier, tag_format_reward)

    t = TaggedAnswerVerifier()
    assert t.verify("<final_answer>$1,200</final_answer>", "1200").value == 1.0
    assert t.verify("<tool_call>{}</tool_call><tool_result>3</tool_result>", "9").value == pytest.approx(0.1)
    assert ExactMatchVerifier().verify("  Paris \n", "paris").passed
    assert tag_format_reward("<think>a</think><final_answer>1</final_answer>") == pytest.approx(0.04)
    assert FormatVerifier("json").verify('{"a": 1}').passed
    p = LastTokenParityVerifier()
    assert p.verify([3, 5, 8]).value in (0.0, 1.0) and p.verify([3, 5, 8]).value != p.verify([3, 5, 7]).value


def test_code_verifier_and_python_tool():
    from rl_project_b200.rollouts.tools.python_executor import PythonExecutorTool, execute_python
    from rl_project_b200.rollouts.verifiers import CodeExecutionVerifier

    assert execute_python("print(6 * 7)").stdout == "42"
    assert PythonExecutorTool()({"code": "raise ValueError('x')"}).startswith("ERROR")
    cv = CodeExecutionVerifier(timeout=10)
    code = "```python\ndef inc(x):\n    return x + 1\n```"
    assert cv.verify(code, "assert inc(1) == 2").value == 1.0
    assert cv.verify(code, "assert inc(1) == 3").value == 0.0  # failed assertion
    assert cv.verify(code, "raise RuntimeError('boom')").value < 0.0  # crash: failure penalty


def test_tool_call_parser():
    from rl_project_b200.rollouts.tools.parser import parse_tagged_output

    out = parse_tagged_output('<think>add</think><tool_call>{"name": "python_executor", "args": {"code": "1"}}'
                              '</tool_call><tool_result>1</tool_result><final_answer>1</final_answer>')
    assert out.tool_call.name == "python_executor" and out.tool_call.args == {"code": "1"}
    assert out.final_answer == "1" and out.thinking == "add" and out.tool_results == ["1"]


def _traj(text, answer="4"):
    return Trajectory(prompt_ids=torch.tensor([1]), response_ids=torch.tensor([2]), response_text=text,
                      task={"answer": answer})


def test_composite_rewards_and_non_finite_rejection():
    from rl_project_b200.rollouts.rewards.composite import (CallableReward, CompositeReward, TagFormatReward,
                                                            VerifierReward, score_trajectories)
    from rl_project_b200.rollouts.verifiers import TaggedAnswerVerifier

    comp = CompositeReward([(VerifierReward(TaggedAnswerVerifier()), 1.0), (TagFormatReward(), 1.0)], clip=(0, 1.01))
    r = comp.score(_traj("<think>x</think><final_answer>4</final_answer>"))
    assert r.value == pytest.approx(1.01) and r.passed
    bad = CallableReward(lambda t: float("nan"), name="nan")
    with pytest.raises(InvalidRewardError):
        score_trajectories(bad, [_traj("x")])
    assert score_trajectories(comp, [_traj("<final_answer>5</final_answer>")]) == [pytest.approx(0.02)]


def test_process_reward_discounts_steps():
    from rl_project_b200.rollouts.rewards.process import ProcessReward, compute_process_reward

    resp = "Step 1: 2 + 2 = 4\nStep 2: check 4 * 1 = 4\n<final_answer>4</final_answer>"
    total, scores = compute_process_reward(resp, "4", gamma=0.5)
    assert scores[-1] == 1.0 and total == pytest.approx(sum(0.5 ** (len(scores) - 2 - i) * s
                                                          for i, s in enumerate(scores[:-1])) + 1.0)
    r = ProcessReward(gamma=0.5).score(_traj(resp))
    assert r.passed and r.components["final"] == 1.0


def test_critic_reward_is_finite_and_ranks():
    from rl_project_b200.rollouts.rewards.critic import heuristic_critic_score

    good = heuristic_critic_score("What is 2+2?", "2 + 2 = 4, so the answer is 4.")
    empty = heuristic_critic_score("What is 2+2?", "")
    assert math.isfinite(good) and math.isfinite(empty) and good >= empty
