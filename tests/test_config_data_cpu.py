"""Configuration and data-layer unit tests (the reference's unit/test_config.py and unit/test_data.py are
the model): presets, validation, manifest round trips, tokenizers, records, corpora, collators, streaming."""
import json

import numpy as np
import pytest
import torch

from rl_project_b200.core.config import (MODEL_PRESETS, DistributedConfig, ExperimentManifest, ModelSpec,
                                         TrainerConfig, capture_runtime_environment, model_spec_from_preset)
from rl_project_b200.core.errors import ConfigError, DatasetError, MalformedRecordError, UnknownPresetError


# ------------------------------------------------------------------ config
def test_every_preset_builds_and_validates():
    for name in MODEL_PRESETS:
        spec = model_spec_from_preset(name)
        spec.validate()
        assert spec.n_embd % spec.n_head == 0 and spec.head_dim > 0
    with pytest.raises(UnknownPresetError):
        model_spec_from_preset("nope")


def test_spec_validation_and_unknown_keys():
    with pytest.raises(ConfigError):
        ModelSpec.from_dict({"n_layer": 2, "n_head": 3, "n_embd": 64})  # heads do not divide the width
    with pytest.raises(ConfigError):
        ModelSpec.from_dict({"n_layer": 2, "not_a_field": 1})
    s = model_spec_from_preset("tiny", vocab_size=77)
    assert ModelSpec.from_dict(s.to_dict()) == s


@pytest.mark.parametrize("suffix", [".yaml", ".toml", ".json"])
def test_manifest_roundtrip_every_format(tmp_path, suffix):
    m = ExperimentManifest.from_dict({
        "name": "rt", "algorithm": "sft", "model_preset": "tiny", "model": {"vocab_size": 96},
        "trainer": {"max_steps": 7, "batch_size": 3, "optimizer": {"learning_rate": 1e-3}},
        "distributed": {"strategy": "fsdp", "timeout_s": 30}, "output_dir": str(tmp_path / "o")})
    p = m.save(tmp_path / f"m{suffix}")
    back = ExperimentManifest.load(p)
    assert back.to_dict() == m.to_dict()
    assert back.trainer.optimizer.learning_rate == 1e-3 and back.model.vocab_size == 96


def test_manifest_rejects_unknown_algorithm_and_keys():
    with pytest.raises(ConfigError):
        ExperimentManifest.from_dict({"name": "x", "algorithm": "not-an-algorithm"})
    with pytest.raises(ConfigError):
        ExperimentManifest.from_dict({"name": "x", "algorithm": "sft", "unknown_section": {}})


def test_trainer_and_distributed_validation():
    with pytest.raises(ConfigError):
        TrainerConfig(batch_size=0).validate()
    with pytest.raises(ConfigError):
        DistributedConfig(strategy="warp-drive").validate()
    with pytest.raises(ConfigError):
        DistributedConfig(fused_comm="maybe").validate()
    DistributedConfig(strategy="hybrid", tensor_parallel_size=2, pipeline_parallel_size=2).validate()


def test_runtime_environment_is_serialisable():
    env = capture_runtime_environment()
    assert json.loads(json.dumps(env)) == env and "torch" in json.dumps(env)


# ------------------------------------------------------------------ data
def test_char_and_byte_tokenizers_roundtrip(tmp_path):
    from rl_project_b200.data.tokenizers import (ByteTokenizer, CharTokenizer, load_tokenizer,
                                                 save_tokenizer_metadata, token_dtype_for)

    tok = CharTokenizer().fit("hello world")
    assert tok.decode(tok.encode("hello world")) == "hello world"
    save_tokenizer_metadata(tok, tmp_path)
    back = load_tokenizer(tmp_path)
    assert back.encode("hello") == tok.encode("hello")
    b = ByteTokenizer()
    assert b.decode(b.encode("héllo ✓")) == "héllo ✓"
    assert token_dtype_for(60000) == np.uint16 and token_dtype_for(70000) == np.uint32


def test_memmap_corpus_windows(tmp_path):
    from rl_project_b200.data.pretraining import MemmapCorpus

    np.arange(500, dtype=np.uint16).tofile(tmp_path / "train.bin")
    c = MemmapCorpus(tmp_path, "train", 16, dtype=np.uint16)
    x, y = c.sample_batch(4, generator=torch.Generator().manual_seed(0))
    assert x.shape == (4, 16) and torch.equal(x[:, 1:], y[:, :-1]) and torch.equal(y - x, torch.ones_like(x))
    windows = list(c)
    assert len(windows) == (500 - 17) // 16 + 1 and torch.equal(windows[1][0], torch.arange(16, 32))
    with pytest.raises(DatasetError):
        MemmapCorpus(tmp_path, "val", 16)


def test_jsonl_records_schema_and_split(tmp_path):
    from rl_project_b200.data.records import ReadReport, SFTRecord, deterministic_split, read_jsonl, write_jsonl

    p = tmp_path / "d.jsonl"
    write_jsonl(p, [SFTRecord("a", "b"), {"prompt": "c", "completion": "d", "id": 3}])
    with p.open("a") as fh:
        fh.write(json.dumps({"prompt": "", "response": "x"}) + "\n")
    with pytest.raises(MalformedRecordError, match=r"d\.jsonl:3"):
        read_jsonl(p, SFTRecord)
    rep = ReadReport()
    recs = read_jsonl(p, SFTRecord, on_error="skip", report=rep)
    assert [r.response for r in recs] == ["b", "d"] and recs[1].meta == {"id": 3}
    assert rep.read == 2 and rep.skipped == 1 and rep.errors[0][0] == 3
    tr, va = deterministic_split(list(range(100)), 0.2, seed=1)
    assert len(va) == 20 and sorted(tr + va) == list(range(100))
    assert deterministic_split(list(range(100)), 0.2, seed=1) == (tr, va)


def test_collate_supervised_masks_the_prompt():
    from rl_project_b200.data.collators import IGNORE_INDEX, collate_supervised

    b = collate_supervised([([1, 2, 3], [4, 5]), ([6], [7, 8, 9])], pad_value=0)
    assert b.input_ids.tolist() == [[1, 2, 3, 4], [6, 7, 8, 9]]
    # prompt positions (all but the last prompt token) and padding are ignored
    assert b.targets.tolist() == [[IGNORE_INDEX, IGNORE_INDEX, 4, 5], [7, 8, 9, IGNORE_INDEX]]
    assert b.attention_mask.tolist() == [[1, 1, 1, 1], [1, 1, 1, 1]]
    assert b.prompt_lengths == [3, 1]


def test_streaming_pack_and_shards(tmp_path):
    from rl_project_b200.data.streaming import ShardedTokenDataset, pack_documents, shard_token_file
    from rl_project_b200.data.tokenizers import ByteTokenizer

    wins = list(pack_documents(["abcdefgh", "ijklmnop", "q"], ByteTokenizer(), 4))
    assert all(x.shape == (4,) and torch.equal(x[1:], y[:-1]) for x, y in wins) and len(wins) >= 3
    np.arange(1000, dtype=np.uint16).tofile(tmp_path / "all.bin")
    paths = shard_token_file(tmp_path / "all.bin", tmp_path / "shards", 4)
    assert len(paths) == 4
    ds0 = ShardedTokenDataset(tmp_path / "shards", 8, shuffle=False, world_size=2, rank=0)
    ds1 = ShardedTokenDataset(tmp_path / "shards", 8, shuffle=False, world_size=2, rank=1)
    assert set(ds0.shard_paths).isdisjoint(ds1.shard_paths) and ds0.total_tokens + ds1.total_tokens == 1000
    x, y = next(iter(ds0))
    assert torch.equal(x[1:], y[:-1])


def test_gsm8k_answer_extraction():
    from rl_project_b200.data.verifiable import extract_gsm8k_answer

    assert extract_gsm8k_answer("She has 3 + 4 = 7.\n#### 1,234") == "1234"
    assert extract_gsm8k_answer("no final answer") == ""
