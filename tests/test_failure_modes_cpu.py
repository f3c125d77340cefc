"""Failure modes on the host (CPU only): each failure surfaces as its typed error
with a hint, or is contained where it happens (a crashing tool becomes an
observation, a bad request fails alone, a crashing verifier scores zero).

The topics follow the reference's ``tests/failure/test_failure_modes.py`` and
``tests/smoke/test_smoke.py``; the assertions are written against this
framework's API.
"""

from __future__ import annotations

import importlib
import json
import pkgutil

import pytest
import torch

import rl_project_b200
from rl_project_b200.core.errors import (ConfigError, DatasetError, DistributedConfigError, ExportError,
                                         ForgelineError, InvalidRewardError, MalformedRecordError, PromotionError,
                                         QuantizationError, RolloutError, ServingError)
from rl_project_b200.core.protocols import Trajectory


def test_dataset_failures(tmp_path):
    from rl_project_b200.data.records import PreferenceRecord, read_jsonl

    with pytest.raises(DatasetError):
        read_jsonl(tmp_path / "missing.jsonl", PreferenceRecord)
    bad = tmp_path / "bad.jsonl"
    bad.write_text(json.dumps({"prompt": "p", "chosen": "c", "rejected": "r"}) + "\n"
                   + json.dumps({"prompt": "p", "chosen": 3, "rejected": "r"}) + "\n")
    with pytest.raises(MalformedRecordError, match="bad.jsonl:2"):
        read_jsonl(bad, PreferenceRecord)
    assert len(read_jsonl(bad, PreferenceRecord, on_error="skip")) == 1


def test_invalid_reward_and_crashing_verifier():
    from rl_project_b200.rollouts.rewards.composite import CallableReward, score_trajectories
    from rl_project_b200.rollouts.verifiers import MathVerifier

    t = Trajectory(prompt_ids=torch.tensor([1]), response_ids=torch.tensor([2]), response_text="x")
    for bad in (float("nan"), float("inf")):
        with pytest.raises(InvalidRewardError):
            score_trajectories(CallableReward(lambda _, v=bad: v), [t])

    class Exploding(MathVerifier):
        @staticmethod
        def extract_answer(text):
            raise RuntimeError("boom")

    r = Exploding().verify("1", "1")
    assert r.passed is False and r.value == 0.0 and "boom" in r.info["error"]


class _Scripted:
    """A policy that answers with fixed text segments, one per generate call."""

    device = torch.device("cpu")
    pad_token_id = 0

    def __init__(self, segments):
        self.segments, self.n = segments, 0

    def encode(self, text):
        return [ord(c) % 128 for c in text]

    def decode(self, ids):
        return self.segments[self.n - 1]

    def generate(self, ids, settings):
        self.n += 1
        return torch.zeros(1, 1, dtype=torch.long)


def test_tool_failures_become_observations():
    from rl_project_b200.rollouts.agent import AgentRolloutConfig, AgentRolloutEngine

    call = '<tool_call>{"name": "python_executor", "args": {"code": "raise ValueError(42)"}}</tool_call>'
    segs = [call, "<final_answer>1</final_answer>"]
    _, blocks, _ = AgentRolloutEngine(_Scripted(list(segs)), AgentRolloutConfig()).run_episode("p")
    assert len(blocks) == 1 and "ValueError" in blocks[0]

    def broken(args):
        raise RuntimeError("tool crashed")

    _, blocks, final = AgentRolloutEngine(_Scripted(list(segs)),
                                          AgentRolloutConfig(tools={"python_executor": broken})).run_episode("p")
    assert "ERROR" in blocks[0] and "tool crashed" in blocks[0]
    assert final.endswith("<final_answer>1</final_answer>")  # the episode went on after the failure


def test_rollout_failures(tiny_spec):
    from rl_project_b200.data.tokenizers import ByteTokenizer
    from rl_project_b200.models.policy import NativePolicy
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine

    class Broken:
        device = torch.device("cpu")
        pad_token_id = 0
        model = None

        def generate(self, *a, **k):
            raise RuntimeError("out of memory")

    with pytest.raises(RolloutError, match="out of memory"):
        RolloutEngine(Broken(), RolloutConfig(engine="generate")).rollout(torch.tensor([1, 2]))
    tok = ByteTokenizer()
    policy = NativePolicy(TransformerLM(tiny_spec.__class__.from_dict({**tiny_spec.to_dict(),
                                                                        "vocab_size": tok.vocab_size})), tok)
    with pytest.raises(RolloutError, match="empty prompt"):
        RolloutEngine(policy, RolloutConfig()).rollout(torch.tensor([], dtype=torch.long))


def test_distributed_misconfiguration():
    from rl_project_b200.core.config import DistributedConfig, ExperimentManifest
    from rl_project_b200.parallel.strategies import validate_distributed_config

    with pytest.raises(DistributedConfigError):
        validate_distributed_config(DistributedConfig(strategy="pipeline_parallel", pipeline_parallel_size=3),
                                    world_size=4)
    with pytest.raises(ConfigError):
        ExperimentManifest.from_dict({"distributed": {"strategy": "fsdp", "tensor_parallel_size": 0}})
    with pytest.raises(ConfigError):
        ExperimentManifest.from_dict({"distributed": {"strategy": "nccl_magic"}})


def test_promotion_failure():
    from rl_project_b200.deployment.promotion import GateRule, PromotionGate

    with pytest.raises(PromotionError, match="reward"):
        PromotionGate([GateRule("reward", min=0.9)]).assert_promotable({"reward": 0.1})


def test_serving_backend_failure():
    from rl_project_b200.serving.api import Router
    from rl_project_b200.serving.backends import EchoBackend

    class Failing(EchoBackend):
        def complete(self, *a, **k):
            raise RuntimeError("backend crashed")

    status, body = Router({"f": Failing("f")}, "f").handle("POST", "/v1/completions", {"prompt": "x"})
    assert status == 500 and "backend crashed" in body["error"]["message"]
    with pytest.raises(ServingError):
        Router({"a": EchoBackend("a")}, "missing")


def test_engine_isolates_failing_sequence(tiny_spec):
    from rl_project_b200.inference.engine import InferenceEngine
    from rl_project_b200.inference.requests import RequestStatus, SamplingParams
    from rl_project_b200.models.transformer.model import TransformerLM

    torch.manual_seed(0)
    eng = InferenceEngine(TransformerLM(tiny_spec), max_batch=4)
    good = eng.submit([1, 2], SamplingParams(max_tokens=3, temperature=0.0))
    bad = eng.submit([tiny_spec.vocab_size + 5], SamplingParams(max_tokens=3, temperature=0.0))
    neg = eng.submit([3, -1], SamplingParams(max_tokens=3, temperature=0.0))
    eng.run_until_idle()
    assert good.status == RequestStatus.FINISHED and len(good.generated_tokens) == 3
    for r in (bad, neg):
        assert r.status == RequestStatus.FAILED and "vocabulary" in r.error
    assert len(eng.allocator.free_blocks) == eng.allocator.max_blocks  # the failed requests gave their blocks back


def test_quantization_and_export_errors(tmp_path, tiny_spec):
    from rl_project_b200.models.quantization.gguf import export_gguf
    from rl_project_b200.models.quantization.nf4 import quantize_nf4
    from rl_project_b200.models.transformer.model import TransformerLM

    with pytest.raises(QuantizationError):
        quantize_nf4(torch.empty(0))
    m = TransformerLM(tiny_spec)
    with pytest.raises(ExportError):
        export_gguf(m.state_dict(), m.spec, tmp_path / "x.gguf", quantize="q3_k")


def test_non_finite_loss_aborts_training(make_ctx):
    from rl_project_b200.training.common.trainer import PostTrainingAlgorithm, Trainer

    class NaNAlgorithm(PostTrainingAlgorithm):
        name = "pretrain"

        def __init__(self):
            self.p = torch.nn.Parameter(torch.ones(1))

        def parameters(self):
            return [self.p]

        def collect(self, step):
            return None

        def loss(self, batch, micro_step, n_micro):
            return (self.p * float("nan")).sum(), {}

    ctx = make_ctx("pretrain", eval_every=0, save_every=0)
    with pytest.raises(ConfigError, match="non-finite loss"):
        Trainer(ctx, NaNAlgorithm()).fit()
    events = [json.loads(x)["event"] for x in (ctx.output_dir / "events.jsonl").read_text().splitlines()]
    assert "run.failed" in events


def test_every_error_has_a_hint():
    import rl_project_b200.core.errors as errors

    for name in errors.__all__:
        cls = getattr(errors, name)
        assert issubclass(cls, ForgelineError)
        assert cls is ForgelineError or cls("x").hint, name


def test_every_module_imports():
    """Every module of the package imports on a machine without a GPU; a module that
    is only an optional extra's front end (Ray) reports the missing extra with its
    typed error instead."""
    from rl_project_b200.core.errors import OptionalDependencyError

    failed = {}
    for mod in pkgutil.walk_packages(rl_project_b200.__path__, "rl_project_b200."):
        if mod.name.endswith("__main__"):
            continue
        try:
            importlib.import_module(mod.name)
        except OptionalDependencyError as exc:
            assert exc.hint, mod.name
        except Exception as exc:  # noqa: BLE001
            failed[mod.name] = repr(exc)
    assert not failed, failed
    assert rl_project_b200.__version__
