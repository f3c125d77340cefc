"""Dashboard data layer and server over a real (tiny) training run."""
from __future__ import annotations

import json
import urllib.request

import pytest
import yaml

from rl_project_b200.cli.main import main
from rl_project_b200.dashboard import DashboardApp, DashboardServer, DashboardSources, snapshot
from rl_project_b200.dashboard import data


@pytest.fixture(scope="module")
def run_root(tmp_path_factory):
    root = tmp_path_factory.mktemp("runs")
    m = {"name": "dash-sft", "algorithm": "sft", "model_preset": "tiny", "model": {"vocab_size": 256, "block_size": 64},
         "data": {"kind": "supervised", "path": "synthetic:addition", "tokenizer": "byte", "max_length": 32},
         "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": 3, "batch_size": 4,
                     "eval_every": 0, "log_every": 1, "checkpoint": {"save_every": 3, "directory": "ckpt"}},
         "output_dir": str(root / "sft")}
    (root / "m.yaml").write_text(yaml.safe_dump(m))
    assert main(["train", str(root / "m.yaml"), "--metrics", "local"]) == 0
    bench = root / "benchmarks" / "rec1"
    bench.mkdir(parents=True)
    (bench / "results.json").write_text(json.dumps({"evidence": "measured", "metrics": {"tok_s": 1.0}}))
    (bench / "summary.md").write_text("# rec1")
    return root


def test_data_layer(run_root):
    runs = data.discover_runs([run_root])
    assert len(runs) == 1 and runs[0]["algorithm"] == "sft" and runs[0]["status"] == "finished"
    d = data.run_detail(runs[0]["path"])
    assert d["series"] and d["checkpoints"] and all(c["valid"] for c in d["checkpoints"])
    assert data.benchmark_records(run_root / "benchmarks")[0]["metrics"] == {"tok_s": 1.0}
    assert data.registry_view(run_root / "none.json")["exists"] is False
    ckpt = d["checkpoints"][-1]["path"]
    info = data.inspect_checkpoint(ckpt, text="12+3=")
    assert info["parameters"] > 0 and info["attention"] and info["activations"] and "inspection_error" not in info
    assert data.downsample([[i, i] for i in range(5000)], 100)[-1] == [4999, 4999]


def test_app_routes_and_guard(run_root):
    src = DashboardSources(runs=[str(run_root)], registry=str(run_root / "reg.json"),
                           benchmarks=str(run_root / "benchmarks"))
    app = DashboardApp(src)
    assert app.handle("/")[0] == 200 and "<html" in app.handle("/")[2]
    st, _, ov = app.handle("/api/overview")
    assert st == 200 and len(ov["runs"]) == 1 and ov["benchmarks"][0]["record"] == "rec1"
    rid = ov["runs"][0]["id"]
    assert app.handle(f"/api/runs/{rid}")[0] == 200 and app.handle("/api/runs/nope")[0] == 404
    ckpt = data.run_detail(ov["runs"][0]["path"])["checkpoints"][0]["path"]
    assert app.handle(f"/api/inspect?checkpoint={ckpt}")[0] == 200
    assert app.handle("/api/inspect?checkpoint=/etc")[0] == 403
    snap = snapshot(src)
    assert rid in snap["run_details"]


def test_http_server(run_root):
    server = DashboardServer(DashboardApp(DashboardSources(runs=[str(run_root)])), port=0).start()
    try:
        with urllib.request.urlopen(server.url + "/health", timeout=30) as r:
            assert json.loads(r.read()) == {"status": "ok"}
        with urllib.request.urlopen(server.url + "/api/runs", timeout=30) as r:
            assert len(json.loads(r.read())) == 1
    finally:
        server.stop()
