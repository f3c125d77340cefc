"""Checkpoint format, validation failures and exact resume."""

import json

import pytest
import torch

from rl_project_b200.checkpoints.manager import CheckpointManager, CheckpointState, load_model_state
from rl_project_b200.checkpoints.validation import assert_compatible, compare_state_shapes, finite_state
from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.core.errors import (CheckpointCorruptError, CheckpointMismatchError, CheckpointNotFoundError,
                                         ForgelineError, IncompatibleStateError)
from rl_project_b200.models.transformer.model import TransformerLM


def _model(v=20):
    return TransformerLM(model_spec_from_preset("tiny", vocab_size=v))


def test_rotation_latest_best_and_roundtrip(tmp_path):
    mgr = CheckpointManager(tmp_path, keep_last=2)
    m = _model()
    for step in (1, 2, 3):
        mgr.save(CheckpointState(model_state=m.state_dict(), step=step, algorithm="sft", model_spec=m.spec.to_dict(),
                                 optimizer_state={"x": step}, trainer_state={"best": 1.0}), is_best=(step == 2))
    names = [p.name for p in mgr.list()]
    assert "step_00000001" not in names and "step_00000003" in names and "best" in names
    assert mgr.find_latest().name == "step_00000003"
    st = CheckpointManager.load(mgr.find_latest(), expected_spec=m.spec.to_dict(), expected_algorithm="sft")
    assert st.step == 3 and st.optimizer_state == {"x": 3} and st.trainer_state["best"] == 1.0
    m2 = _model()
    load_model_state(m2, st.model_state)
    assert torch.equal(m2.lm_head.weight, m.lm_head.weight)
    man = json.loads((mgr.find_latest() / "manifest.json").read_text())
    assert man["complete"] and "model.pt" in man["files"] and man["format_version"] == 1


def test_async_save(tmp_path):
    mgr = CheckpointManager(tmp_path, async_save=True)
    mgr.save(CheckpointState(model_state={"w": torch.zeros(2)}, step=1), name="a")
    mgr.wait()
    assert (tmp_path / "a" / "manifest.json").exists()


def test_compile_prefix_and_shape_checks():
    m = _model()
    load_model_state(_model(), {f"_orig_mod.{k}": v for k, v in m.state_dict().items()})
    other = _model(30)
    assert compare_state_shapes(other, m.state_dict())["mismatched"]
    with pytest.raises(IncompatibleStateError):
        assert_compatible(other, m.state_dict())
    with pytest.raises(IncompatibleStateError):
        load_model_state(other, m.state_dict())
    assert finite_state(m.state_dict()) and not finite_state({"w": torch.tensor([float("nan")])})


@pytest.fixture
def saved(tmp_path):
    m = _model()
    p = CheckpointManager(tmp_path).save(CheckpointState(model_state=m.state_dict(), step=5, algorithm="sft",
                                                         model_spec=m.spec.to_dict()))
    return p, m


def test_every_error_has_a_hint():
    for cls in ForgelineError.__subclasses__():
        assert cls("x").hint


def test_missing_corrupt_truncated_incomplete(saved, tmp_path):
    path, _ = saved
    with pytest.raises(CheckpointNotFoundError):
        CheckpointManager.load(tmp_path / "nope")
    man = json.loads((path / "manifest.json").read_text())
    with open(path / "model.pt", "r+b") as fh:
        fh.truncate(10)
    with pytest.raises(CheckpointCorruptError, match="truncated"):
        CheckpointManager.load(path)
    (path / "model.pt").unlink()
    with pytest.raises(CheckpointCorruptError, match="missing model.pt"):
        CheckpointManager.load(path)
    man["complete"] = False
    (path / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(CheckpointCorruptError, match="incomplete"):
        CheckpointManager.load(path)
    (path / "manifest.json").write_text("{broken")
    with pytest.raises(CheckpointCorruptError):
        CheckpointManager.load(path)
    (path / "manifest.json").unlink()
    with pytest.raises(CheckpointCorruptError, match="no manifest"):
        CheckpointManager.load(path)


def test_tmp_dirs_ignored_and_mismatch(saved, tmp_path):
    path, _ = saved
    (tmp_path / "step_00000099.tmp").mkdir()
    assert CheckpointManager(tmp_path).find_latest().name == path.name
    with pytest.raises(CheckpointMismatchError):
        CheckpointManager.load(path, expected_spec={"n_layer": 12})
    with pytest.raises(CheckpointMismatchError):
        CheckpointManager.load(path, expected_algorithm="dpo")


def test_resume_matches_uninterrupted(make_ctx, cspec, corpus_dir):
    from rl_project_b200.data.pretraining import MemmapCorpus
    from rl_project_b200.training import PretrainAlgorithm, PretrainConfig, Trainer

    def build(run):
        torch.manual_seed(0)
        alg = PretrainAlgorithm(TransformerLM(cspec), MemmapCorpus(corpus_dir, "train", 64), PretrainConfig(batch_size=4))
        return alg, make_ctx("pretrain", max_steps=6, eval_every=0, save_every=3, run=run)

    alg, ctx = build("full")
    full = Trainer(ctx, alg)
    full.fit()
    ref_losses = [r.loss for r in full.history]

    alg, ctx = build("part")
    part = Trainer(ctx, alg)
    part.fit(max_steps=3)
    alg2, ctx2 = build("part")
    resumed = Trainer(ctx2, alg2)
    assert resumed.resume()
    assert resumed.step == 3
    resumed.fit()
    got = [r.loss for r in resumed.history]
    assert all(abs(a - b) < 1e-5 for a, b in zip(ref_losses[3:], got)), (ref_losses, got)
