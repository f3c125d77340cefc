"""Observability, topology and orchestration-config unit tests (CPU only).

Covers the topics of the reference's ``tests/unit/test_observability_cli.py``,
``tests/unit/test_distributed.py`` and ``tests/unit/test_orchestration_config.py``
against this framework's API: the JSONL metrics sink, the structured logger,
tracer spans and per-parameter gradient norms, the mesh rank layout, the 1F1B
step order, topology validation, strategy construction and the Ray settings
of a manifest.
"""

from __future__ import annotations

import io
import json
import logging
import subprocess
import sys

import pytest
import torch

from rl_project_b200.core.config import DistributedConfig, ExperimentManifest
from rl_project_b200.core.errors import ConfigError, DistributedConfigError
from rl_project_b200.observability.logging import StructuredLogger
from rl_project_b200.observability.metrics import (LocalJsonlMetricsSink, NoOpMetricsSink, build_metrics_sink,
                                                   gradient_norms, perf_metrics)
from rl_project_b200.observability.tracing import Tracer
from rl_project_b200.orchestration.config import RayConfig, validate_orchestration
from rl_project_b200.parallel.pipeline import schedule_1f1b
from rl_project_b200.parallel.runtime import validate_topology
from rl_project_b200.parallel.strategies import build_strategy, validate_distributed_config
from rl_project_b200.parallel.topology import ParallelMesh


# --------------------------------------------------------------------------- observability


def test_local_metrics_sink_round_trip(tmp_path):
    sink = build_metrics_sink("local", output_dir=tmp_path, run_name="r")
    assert isinstance(sink, LocalJsonlMetricsSink)
    sink.log({"loss": 2.5, "lr": torch.tensor(1e-3)}, step=1)
    sink.log({"loss": 2.0}, step=2)
    sink.event("checkpoint", {"path": "ckpt/2"})
    assert sink.increment("restarts") == 1 and sink.increment("restarts", 2) == 3
    assert sink.latest("loss") == 2.0 and sink.series("loss") == [2.5, 2.0]
    assert sink.latest("missing") is None
    rows = [json.loads(x) for x in (tmp_path / "metrics.jsonl").read_text().splitlines()]
    assert [r["step"] for r in rows] == [1, 2]
    assert rows[0]["lr"] == pytest.approx(1e-3)  # tensors become plain numbers
    ev = [json.loads(x) for x in (tmp_path / "events.jsonl").read_text().splitlines()]
    assert ev[0]["event"] == "checkpoint" and ev[0]["path"] == "ckpt/2" and ev[0]["step"] == 2
    assert isinstance(build_metrics_sink("none"), NoOpMetricsSink)
    with pytest.raises(ConfigError):
        build_metrics_sink("nope")


def test_perf_metrics():
    m = perf_metrics(tokens=1000, seconds=0.5, n_params=10**9, peak_tflops=1000.0, world_size=2)
    assert m["perf/tokens_per_s"] == 2000.0
    assert m["perf/model_tflops"] == pytest.approx(6 * 1e9 * 2000 / 1e12)
    assert m["perf/mfu"] == pytest.approx(m["perf/model_tflops"] / 2000.0)
    assert perf_metrics(10, 0.0, 1) == {}


@pytest.mark.parametrize("fmt", ["text", "json"])
def test_structured_logger(monkeypatch, fmt):
    monkeypatch.setenv("FORGELINE_LOG_FORMAT", fmt)
    buf = io.StringIO()
    handler = logging.StreamHandler(buf)
    log = StructuredLogger("forgeline.test_structured")
    log._log.addHandler(handler)
    log.setLevel(logging.INFO)
    try:
        log.info("step_done", step=3, loss=torch.tensor(1.5), tags=("a", "b"))
        log.debug("hidden", x=1)  # below the level: nothing written
    finally:
        log._log.removeHandler(handler)
    lines = buf.getvalue().strip().splitlines()
    assert len(lines) == 1
    if fmt == "json":
        rec = json.loads(lines[0])
        assert rec["event"] == "step_done" and rec["step"] == 3 and rec["loss"] == 1.5
        assert rec["tags"] == ["a", "b"] and rec["logger"] == "forgeline.test_structured"
    else:
        assert lines[0] == "step_done step=3 loss=1.5 tags=['a', 'b']"


def test_tracer_and_grad_norms():
    tr = Tracer(keep=2)
    for i in range(3):
        with tr.span("step", i=i) as s:
            assert s.attributes == {"i": i}
    with tr.span("eval"):
        pass
    s = tr.summary()
    assert s["step"]["count"] == 3 and s["eval"]["count"] == 1  # aggregates cover every span
    assert len(tr.spans) == 2  # only the most recent ``keep`` spans are kept
    assert s["step"]["mean_ms"] == pytest.approx(s["step"]["total_ms"] / 3)
    assert all(d >= 0 for d in tr.durations("step"))

    model = torch.nn.Sequential()
    model.add_module("wte", torch.nn.Embedding(5, 3))
    model.add_module("mid", torch.nn.Linear(3, 3))
    model.add_module("lm_head", torch.nn.Linear(3, 5, bias=False))
    model.mid.bias.requires_grad_(False)
    out = model.lm_head(model.mid(model.wte(torch.tensor([0, 1, 2]))))
    out.square().sum().backward()
    g = gradient_norms(model)
    total = torch.cat([p.grad.flatten() for p in model.parameters() if p.grad is not None]).norm()
    assert g["grad_norm/total"] == pytest.approx(float(total), rel=1e-5)
    assert set(g) == {"grad_norm/total", "grad_norm/wte.weight", "grad_norm/lm_head.weight"}
    assert g["grad_norm/wte.weight"] == pytest.approx(float(model.wte.weight.grad.norm()), rel=1e-6)


# --------------------------------------------------------------------------- distributed layout


def test_mesh_layout():
    # rank = dp * (pp * tp) + pp * tp + tp: tensor-parallel ranks adjacent, then stages, then replicas
    mesh = ParallelMesh(world_size=8, tp_size=2, pp_size=2, rank=5)
    assert mesh.dp_size == 2
    assert mesh.coords() == {"dp": 1, "pp": 0, "tp": 1}
    for r in range(8):
        c = mesh.coords(r)
        assert mesh.rank_of(c["dp"], c["pp"], c["tp"]) == r
    assert mesh.tp_ranks() == [4, 5]
    assert mesh.pp_ranks() == [5, 7]
    assert mesh.dp_ranks() == [1, 5]
    assert mesh.is_first_stage and not mesh.is_last_stage
    assert mesh.prev_stage is None and mesh.next_stage == 7
    last = ParallelMesh(world_size=8, tp_size=2, pp_size=2, rank=7)
    assert last.prev_stage == 5 and last.next_stage is None and last.is_last_stage
    d = mesh.describe()
    assert (d["tp"], d["pp"], d["dp"], d["tp_rank"], d["dp_rank"]) == (2, 2, 2, 1, 1)


def test_expert_groups_partition_a_stage():
    mesh = ParallelMesh(world_size=8, tp_size=1, pp_size=1, ep_size=4, rank=6)
    assert mesh.ep_ranks() == [4, 5, 6, 7]
    with pytest.raises(DistributedConfigError):
        ParallelMesh(world_size=8, tp_size=1, pp_size=1, ep_size=3)


def test_schedule_orders():
    # 4 micro-batches on 4 stages: stage s warms up with 3 - s forwards, ends with as many backwards
    for n_stages in (1, 2, 4):
        for stage in range(n_stages):
            steps = schedule_1f1b(4, stage, n_stages)
            assert sorted(steps) == sorted([("F", i) for i in range(4)] + [("B", i) for i in range(4)])
            done_f = set()
            for kind, i in steps:  # a backward never precedes its own forward; each kind keeps order
                if kind == "F":
                    done_f.add(i)
                else:
                    assert i in done_f
            assert [i for k, i in steps if k == "F"] == list(range(4))
            assert [i for k, i in steps if k == "B"] == list(range(4))
    assert schedule_1f1b(4, 0, 4)[:4] == [("F", 0), ("F", 1), ("F", 2), ("F", 3)]
    assert schedule_1f1b(4, 3, 4)[:4] == [("F", 0), ("B", 0), ("F", 1), ("B", 1)]
    assert schedule_1f1b(2, 0, 4) == [("F", 0), ("F", 1), ("B", 0), ("B", 1)]  # fewer micro-batches than stages


def test_topology_validation():
    assert validate_topology(8, 2, 2) == 2
    assert validate_topology(8, 1, 1, 8) == 8
    for bad in ((8, 3, 1), (8, 0, 1), (6, 1, 1, 4)):
        with pytest.raises(DistributedConfigError):
            validate_topology(*bad)
    topo = validate_distributed_config(DistributedConfig(strategy="hybrid", tensor_parallel_size=2,
                                                         pipeline_parallel_size=2), world_size=8)
    assert topo == {"world_size": 8, "tensor_parallel": 2, "pipeline_parallel": 2, "expert_parallel": 1,
                    "data_parallel": 2}
    with pytest.raises(DistributedConfigError):  # a tensor-parallel strategy with tp = 1
        validate_distributed_config(DistributedConfig(strategy="tensor_parallel"), world_size=2)
    with pytest.raises(ConfigError):  # accepted by the schema, refused instead of silently ignored
        DistributedConfig(strategy="fsdp", context_parallel_size=2).validate()


def test_build_strategy_and_env(monkeypatch):
    cases = {"single": {}, "ddp": {}, "fsdp": {}, "zero2": {}, "hybrid": {},
             "tensor_parallel": {"tensor_parallel_size": 2}, "pipeline_parallel": {"pipeline_parallel_size": 2},
             "expert_parallel": {"expert_parallel_size": 2}}
    for name, kw in cases.items():
        assert build_strategy(DistributedConfig(strategy=name, **kw)).name == name
    with pytest.raises((ConfigError, DistributedConfigError)):
        build_strategy(DistributedConfig(strategy="megatron"))
    # validate_distributed_config reads the world size from the launcher's environment
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "4")
    topo = validate_distributed_config(DistributedConfig(strategy="fsdp"))
    assert topo["world_size"] == 4 and topo["data_parallel"] == 4


# --------------------------------------------------------------------------- orchestration settings


def test_ray_config_validation():
    RayConfig().validate()
    RayConfig(backend="threads", rollout_workers=4, placement_strategy="SPREAD").validate()
    for bad in (dict(backend="slurm"), dict(address="ray://h:10001", num_cpus=4), dict(rollout_workers=-1),
                dict(gpus_per_worker=-0.5), dict(placement_strategy="RANDOM"), dict(max_restarts=-2),
                dict(max_call_retries=-1)):
        with pytest.raises(ConfigError):
            RayConfig(**bad).validate()
    with pytest.raises(ConfigError):
        RayConfig.from_dict({"rollout_workers": 2, "workers": 3})  # unknown key
    validate_orchestration({})
    validate_orchestration({"type": "local"})
    with pytest.raises(ConfigError):
        validate_orchestration({"type": "kubernetes"})
    with pytest.raises(ConfigError):
        validate_orchestration({"type": "ray", "placement_strategy": "NOPE"})


@pytest.mark.parametrize("suffix", [".yaml", ".json", ".toml"])
def test_manifest_orchestration_field_roundtrip(tmp_path, suffix):
    orch = {"type": "ray", "rollout_workers": 2, "reward_workers": 1, "backend": "threads",
            "placement_strategy": "PACK", "max_restarts": 0}
    m = ExperimentManifest.from_dict({"name": "orch", "algorithm": "grpo", "orchestration": orch})
    path = m.save(tmp_path / f"m{suffix}")
    back = ExperimentManifest.load(path)
    assert back.orchestration == orch
    with pytest.raises(ConfigError):
        ExperimentManifest.from_dict({"orchestration": {"type": "ray", "rollout_workers": -3}})


def test_core_import_does_not_import_ray():
    code = ("import sys; import rl_project_b200, rl_project_b200.core.config, rl_project_b200.orchestration.config; "
            "print('ray' in sys.modules)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "False"


def test_nvtx_ranges_are_off_by_default_and_switchable():
    from rl_project_b200.observability import tracing

    calls = []

    @tracing.nvtx_annotate("rlb/test")
    def f(x):
        calls.append(x)
        return x + 1

    before = tracing.nvtx_enabled()
    try:
        tracing.set_nvtx(True)  # without CUDA the range is still a no-op, the call goes through
        assert f(1) == 2
        with tracing.nvtx_range("rlb/block"):
            calls.append("block")
    finally:
        tracing.set_nvtx(before)
    assert f(2) == 3 and calls == [1, "block", 2]
    assert f.__name__ == "f"


def test_trainer_logs_perf_metrics(make_ctx, cspec, corpus_dir):
    import json as _json

    from rl_project_b200.data.pretraining import MemmapCorpus
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    ctx = make_ctx("pretrain", max_steps=3, eval_every=0, save_every=0)
    model = TransformerLM(cspec)
    alg = PretrainAlgorithm(model, MemmapCorpus(corpus_dir, "train", cspec.block_size), PretrainConfig(batch_size=2))
    Trainer(ctx, alg).fit()
    rows = [_json.loads(x) for x in (ctx.output_dir / "metrics.jsonl").read_text().splitlines()]
    perf = [r for r in rows if "perf/tokens_per_s" in r]
    assert len(perf) == 3 and all(r["perf/tokens_per_s"] > 0 for r in perf)
    n = sum(p.numel() for p in model.parameters())
    r = perf[-1]
    assert r["perf/model_tflops"] == pytest.approx(6 * n * r["perf/tokens_per_s"] / 1e12, rel=1e-6)


def test_tokens_in_reads_batch_shapes():
    from types import SimpleNamespace

    from rl_project_b200.core.protocols import Trajectory
    from rl_project_b200.training.common.trainer import PostTrainingAlgorithm

    tokens_in = PostTrainingAlgorithm.tokens_in
    assert tokens_in(None, torch.zeros(3, 7)) == 21
    assert tokens_in(None, (torch.zeros(2, 5), torch.zeros(2, 5))) == 10
    assert tokens_in(None, {"input_ids": torch.zeros(4, 4)}) == 16
    t = Trajectory(prompt_ids=torch.zeros(6, dtype=torch.long), response_ids=torch.zeros(3, dtype=torch.long))
    groups = [SimpleNamespace(trajectories=[t, t]), SimpleNamespace(trajectories=[t])]
    assert tokens_in(None, groups) == 3 * 9
    assert tokens_in(None, "opaque") == 0
