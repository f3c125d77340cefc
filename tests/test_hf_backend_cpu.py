"""The HuggingFace backend on CPU with a tiny offline Llama (the reference's
integration/test_huggingface_backend.py is the model): log-probs, values, generation, checkpoint state,
the optional-dependency error for LoRA without peft, and an SFT step through the manifest factory."""
import importlib.util

import pytest
import torch

transformers = pytest.importorskip("transformers")
pytest.importorskip("tokenizers")


@pytest.fixture(scope="module")
def tiny_llama(tmp_path_factory):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import LlamaConfig, LlamaForCausalLM, PreTrainedTokenizerFast

    root = tmp_path_factory.mktemp("hf") / "tiny-llama"
    symbols = ["<pad>", "<eos>"] + [chr(c) for c in range(32, 127)] + ["\n"]
    tok = Tokenizer(models.WordLevel(vocab={s: i for i, s in enumerate(symbols)}, unk_token="<pad>"))
    tok.pre_tokenizer = pre_tokenizers.Split(pattern="", behavior="isolated")
    tok.decoder = decoders.Fuse()  # characters back to text without separators
    PreTrainedTokenizerFast(tokenizer_object=tok, pad_token="<pad>", eos_token="<eos>").save_pretrained(root)
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=len(symbols), hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=2, max_position_embeddings=256, pad_token_id=0,
                      eos_token_id=1)
    LlamaForCausalLM(cfg).save_pretrained(root)
    return str(root)


def _policy(path, **kw):
    from rl_project_b200.models.hf_policy import HFPolicy

    return HFPolicy(path, use_lora=False, device_map=None, gradient_checkpointing=False, **kw)


def test_logprobs_values_generation_and_state(tiny_llama):
    from rl_project_b200.core.protocols import GenerationSettings

    pol = _policy(tiny_llama, value_head=True)
    p = torch.tensor([pol.encode("1+1=")])
    r = torch.tensor([pol.encode("2!")])
    lp = pol.logprobs(p, r)
    full = torch.cat([p, r], 1)
    logits = pol.model(input_ids=full).logits.float()
    want = torch.log_softmax(logits[:, :-1], -1).gather(-1, full[:, 1:, None])[..., 0][:, p.shape[1] - 1:]
    torch.testing.assert_close(lp.float(), want, atol=1e-4, rtol=1e-4)
    lp2, v = pol.logprobs_and_values(p, r)
    assert v.shape == (1,) and torch.isfinite(v).all()
    torch.testing.assert_close(lp2.float(), lp.float())
    out = pol.generate(p, GenerationSettings(max_new_tokens=3, temperature=0.0))
    assert out.shape[0] == 1 and out.shape[1] >= 1
    st = pol.state_for_checkpoint()
    other = _policy(tiny_llama, value_head=True)
    with torch.no_grad():
        for q in other.model.parameters():
            q.add_(1.0)
    other.load_checkpoint_state(st)
    torch.testing.assert_close(other.logprobs(p, r), lp)
    assert pol.decode(pol.encode("abc")) == "abc"


@pytest.mark.skipif(importlib.util.find_spec("peft") is not None, reason="peft is installed")
def test_lora_without_peft_reports_the_optional_dependency(tiny_llama):
    from rl_project_b200.core.errors import OptionalDependencyError
    from rl_project_b200.models.hf_policy import HFPolicy

    with pytest.raises(OptionalDependencyError):
        HFPolicy(tiny_llama, use_lora=True, device_map=None, gradient_checkpointing=False)


def test_sft_step_through_the_manifest(tiny_llama, tmp_path):
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    m = ExperimentManifest.from_dict({
        "name": "hf-sft", "algorithm": "sft", "output_dir": str(tmp_path / "o"),
        "backend": {"type": "huggingface", "model_name": tiny_llama, "use_lora": False,
                    "gradient_checkpointing": False},
        "data": {"kind": "supervised", "path": "synthetic:addition", "max_length": 32, "extra": {"n_tasks": 16}},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": 2, "batch_size": 4,
                    "eval_every": 0, "log_every": 0, "checkpoint": {"save_every": 0}}})
    ctx = RunContext.create(m, metrics_backend="none")
    alg = build_algorithm(m, ctx)
    tr = Trainer(ctx, alg)
    losses = [tr.train_step().loss for _ in range(2)]
    assert all(torch.isfinite(torch.tensor(losses)))


def test_entropy_and_frozen_reference(tiny_llama):
    pol = _policy(tiny_llama)
    p = torch.tensor([pol.encode("ab")])
    r = torch.tensor([pol.encode("cd")])
    lp, ent = pol.logprobs_with_entropy(p, r)
    torch.testing.assert_close(lp.float(), pol.logprobs(p, r).float(), atol=1e-5, rtol=1e-5)
    assert ent.shape == lp.shape and (ent > 0).all()
    pol.with_frozen_reference()
    with torch.no_grad():
        for q in pol.model.parameters():
            q.add_(0.05)
    with pol.reference():
        ref_lp = pol.logprobs(p, r)
    assert (ref_lp - pol.logprobs(p, r)).abs().max() > 1e-4  # the reference kept the initial weights
    torch.testing.assert_close(ref_lp.float(), lp.float(), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("algorithm", ["dpo", "grpo", "ppo"])
def test_preference_and_rl_steps_on_the_hf_backend(tiny_llama, tmp_path, algorithm):
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    import json

    pref = tmp_path / "pref.jsonl"
    pref.write_text("".join(json.dumps({"prompt": f"{i}+1=", "chosen": str(i + 1), "rejected": str(i + 2)}) + "\n"
                            for i in range(8)))
    data = {"dpo": {"kind": "preference", "path": str(pref), "max_length": 32},
            "grpo": {"kind": "verifiable", "path": "synthetic:addition", "extra": {"n_tasks": 8}},
            "ppo": {"kind": "verifiable", "path": "synthetic:addition", "extra": {"n_tasks": 8}}}[algorithm]
    params = {"dpo": {}, "grpo": {"group_size": 2, "prompts_per_step": 2,
                                  "rollout": {"max_new_tokens": 4, "engine": "generate"}},
              "ppo": {"rollout": {"max_new_tokens": 4, "engine": "generate"}, "prompts_per_step": 2}}[algorithm]
    m = ExperimentManifest.from_dict({
        "name": f"hf-{algorithm}", "algorithm": algorithm, "output_dir": str(tmp_path / "o"),
        "backend": {"type": "huggingface", "model_name": tiny_llama, "use_lora": False,
                    "gradient_checkpointing": False},
        "data": data, "reward": {"type": "verifier", "verifier": "math"}, "algorithm_params": params,
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": 1, "batch_size": 2,
                    "eval_every": 0, "log_every": 0, "checkpoint": {"save_every": 0}}})
    ctx = RunContext.create(m, metrics_backend="none")
    res = Trainer(ctx, build_algorithm(m, ctx)).train_step()
    assert torch.isfinite(torch.tensor(res.loss))
