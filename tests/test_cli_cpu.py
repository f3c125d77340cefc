"""The command-line interface end to end on CPU: train -> checkpoint -> generate /
evaluate / export -> registry life cycle."""
from __future__ import annotations

import json

import pytest
import yaml

from rl_project_b200.cli.main import build_parser, main


def _manifest(tmp_path):
    m = {"name": "cli-sft", "algorithm": "sft", "model_preset": "tiny",
         "model": {"vocab_size": 256, "block_size": 64},
         "data": {"kind": "supervised", "path": "synthetic:addition", "tokenizer": "byte", "max_length": 32,
                  "extra": {"n_tasks": 64}},
         "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": 4, "batch_size": 4,
                     "eval_every": 0, "log_every": 1, "checkpoint": {"save_every": 2, "directory": "ckpt"}},
         "output_dir": str(tmp_path / "run")}
    path = tmp_path / "m.yaml"
    path.write_text(yaml.safe_dump(m))
    return path


def test_parser_has_all_commands():
    sub = next(a for a in build_parser()._actions if a.dest == "command")
    assert set(sub.choices) == {"presets", "validate", "data", "train", "generate", "evaluate", "serve", "export",
                                "registry", "rlaif", "dashboard", "allocation", "synthesis-ppo"}


def test_train_generate_evaluate_export_registry(tmp_path, capsys):
    mpath = _manifest(tmp_path)
    assert main(["validate", str(mpath), "--world-size", "1"]) == 0
    assert json.loads(capsys.readouterr().out)["topology"]["data_parallel"] == 1
    assert main(["train", str(mpath), "--metrics", "none", "--set", "trainer.optimizer.learning_rate=0.003"]) == 0
    summary = json.loads(capsys.readouterr().out)
    assert summary["step"] == 4 if "step" in summary else True
    ckpts = sorted((tmp_path / "run").rglob("manifest.json"))
    assert ckpts, "training wrote no checkpoint"
    ckpt = str(ckpts[-1].parent)

    assert main(["generate", "--checkpoint", ckpt, "--prompt", "1+2=", "--max-tokens", "4", "--temperature", "0",
                 "--device", "cpu"]) == 0
    capsys.readouterr()
    out = tmp_path / "eval.json"
    assert main(["evaluate", "--checkpoint", ckpt, "--device", "cpu", "--suites", "gsm8k", "arc", "--offline",
                 "--max-tokens", "4", "--output", str(out)]) == 0
    rows = json.loads(capsys.readouterr().out)
    assert [r["suite"] for r in rows] == ["benchmark/gsm8k", "benchmark/arc"] and out.exists()
    gguf = tmp_path / "m.gguf"
    assert main(["export", "--checkpoint", ckpt, "--output", str(gguf), "--quantize", "q8_0"]) == 0
    assert gguf.stat().st_size > 0
    capsys.readouterr()

    reg = str(tmp_path / "reg.json")
    gate = tmp_path / "gate.yaml"
    gate.write_text(yaml.safe_dump({"rules": [{"metric": "benchmark/gsm8k/accuracy", "min": 0.0}]}))
    ids = []
    for v in ("1", "2"):
        assert main(["registry", "--registry", reg, "register", "--name", "m", "--version", v, "--algorithm", "sft",
                     "--checkpoint", ckpt, "--metrics-file", str(out)]) == 0
        ids.append(json.loads(capsys.readouterr().out)["registered"])
        assert main(["registry", "--registry", reg, "promote", "--id", ids[-1], "--to", "champion",
                     "--gate", str(gate)]) == 0
        capsys.readouterr()
    assert main(["registry", "--registry", reg, "rollback", "--name", "m"]) == 0
    assert json.loads(capsys.readouterr().out)["champion"] == "m:1"
    assert main(["registry", "--registry", reg, "list"]) == 0
    states = {r["key"]: r["state"] for r in json.loads(capsys.readouterr().out)}
    assert states == {"m:1": "champion", "m:2": "retired"}


def test_presets_and_rlaif(tmp_path, capsys):
    assert main(["presets"]) == 0
    assert any(r["preset"] == "bl_dense_1b" for r in json.loads(capsys.readouterr().out))
    out = tmp_path / "pairs.jsonl"
    assert main(["rlaif", "pairwise", "--output", str(out), "--n-prompts", "3", "--candidates", "2"]) == 0
    capsys.readouterr()
    assert out.exists() or any(tmp_path.iterdir())


def test_bad_manifest_reports_error(tmp_path, capsys):
    bad = tmp_path / "bad.yaml"
    bad.write_text(yaml.safe_dump({"name": "x", "algorithm": "nope"}))
    assert main(["validate", str(bad)]) == 1
    assert "error" in capsys.readouterr().err


def test_data_prepare_shard_and_validate(tmp_path, capsys):
    import numpy as np

    text = tmp_path / "corpus.txt"
    text.write_text("the quick brown fox jumps over the lazy dog. " * 200)
    out = tmp_path / "prepared"
    assert main(["data", "prepare", "--input", str(text), "--output", str(out), "--tokenizer", "char",
                 "--val-fraction", "0.1"]) == 0
    capsys.readouterr()
    assert (out / "train.bin").exists() and (out / "val.bin").exists() and (out / "meta.pkl").exists()
    n_train = (out / "train.bin").stat().st_size
    n_val = (out / "val.bin").stat().st_size
    assert n_val > 0 and 0.05 < n_val / (n_train + n_val) < 0.15  # the validation tail

    shards = tmp_path / "shards"
    assert main(["data", "shard", "--input", str(out / "train.bin"), "--output", str(shards), "--n-shards", "3"]) == 0
    paths = json.loads(capsys.readouterr().out)
    assert len(paths) == 3
    whole = np.fromfile(out / "train.bin", dtype=np.uint16)
    joined = np.concatenate([np.fromfile(p, dtype=np.uint16) for p in sorted(paths)])
    assert np.array_equal(joined, whole)  # shards partition the token stream in order

    jl = tmp_path / "sft.jsonl"
    jl.write_text(json.dumps({"prompt": "a", "response": "b"}) + "\n" + json.dumps({"prompt": 3}) + "\n")
    assert main(["data", "validate", "--input", str(jl), "--kind", "supervised"]) == 0
    rep = json.loads(capsys.readouterr().out)
    assert rep["valid"] == 1 and rep["skipped"] == 1 and rep["errors"][0][0] == 2  # (line, reason)
