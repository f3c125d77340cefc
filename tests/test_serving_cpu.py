"""Serving: router status mapping, schemas, engine backend, HTTP server (CPU)."""
from __future__ import annotations

import json
import urllib.error
import urllib.request

import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.data.tokenizers import CharTokenizer
from rl_project_b200.inference import InferenceEngine
from rl_project_b200.models.transformer.model import TransformerLM
from rl_project_b200.serving import EchoBackend, EngineBackend, Router, ServingServer


def test_router_routes_and_status_codes():
    echo, down = EchoBackend("echo"), EchoBackend("down")
    down.disable()
    r = Router({"echo": echo, "down": down}, default_model="echo")
    assert r.handle("GET", "/health")[1]["status"] == "ok"
    assert {m["id"] for m in r.handle("GET", "/v1/models")[1]["data"]} == {"echo", "down"}
    st, out = r.handle("POST", "/v1/completions", {"prompt": "abcdef", "max_tokens": 3})
    assert st == 200 and out["choices"][0]["text"] == "fed" and out["usage"]["total_tokens"] == 9
    st, out = r.handle("POST", "/v1/chat/completions", {"messages": [{"role": "user", "content": "hi"}]})
    assert st == 200 and out["object"] == "chat.completion"
    assert r.handle("POST", "/v1/completions", {"prompt": ""})[0] == 400
    assert r.handle("POST", "/v1/completions", {"prompt": "x", "temperature": -1})[0] == 400
    assert r.handle("POST", "/v1/chat/completions", {"messages": [{"role": "robot", "content": "x"}]})[0] == 400
    assert r.handle("POST", "/v1/completions", {"prompt": "x", "model": "nope"})[0] == 400
    assert r.handle("POST", "/v1/completions", {"prompt": "x", "model": "down"})[0] == 503
    assert r.handle("GET", "/nope")[0] == 404
    st, stream = r.handle("POST", "/v1/completions", {"prompt": "abc", "stream": True})
    lines = list(stream)
    assert lines[-1] == "data: [DONE]\n\n" and json.loads(lines[0][6:])["choices"][0]["text"] == "c"
    m = r.handle("GET", "/metrics")[1]
    assert m["requests_total"] == 3 and m["errors_total"] == 5


def test_route_fn_selects_backend():
    a, b = EchoBackend("a"), EchoBackend("b")
    r = Router({"a": a, "b": b}, default_model="a", route_fn=lambda rid, req: "b" if rid.startswith("x") else "a")
    out = r.handle("POST", "/v1/completions", {"prompt": "q", "request_id": "xyz"})[1]
    assert out["forgeline"]["backend"] == "b"


@pytest.fixture
def engine_backend():
    torch.manual_seed(0)
    tok = CharTokenizer.ascii()
    spec = model_spec_from_preset("tiny", vocab_size=tok.vocab_size)
    model = TransformerLM(spec).eval()
    eng = InferenceEngine(model, max_batch=4)
    be = EngineBackend("tiny", eng, tok, background=True)
    yield be, tok, model
    be.close()


def test_engine_backend_complete_stream_and_stop(engine_backend):
    from rl_project_b200.inference import SamplingParams

    be, tok, model = engine_backend
    p = SamplingParams(max_tokens=10, temperature=0.0, top_k=None)
    full = be.complete("hello", p)
    ids = torch.tensor([tok.encode("hello")])
    ref = tok.decode(model.generate(ids, 10, temperature=0.0, use_cache=False)[0, ids.shape[1]:].tolist())
    assert full.text == ref and full.completion_tokens == 10
    assert "".join(be.stream("hello", p)) == ref
    if len(ref) > 3:
        stop = ref[2:4]
        cut = be.complete("hello", p, stop=[stop])
        assert cut.text == ref[: ref.find(stop)] and cut.finish_reason == "stop"
        assert "".join(be.stream("hello", p, stop=[stop])) == ref[: ref.find(stop)]


def test_http_server_end_to_end(engine_backend):
    be, _, _ = engine_backend
    server = ServingServer(Router({"tiny": be, "echo": EchoBackend()}, default_model="tiny"), port=0)
    server.start()
    base = f"http://127.0.0.1:{server.port}"
    try:
        with urllib.request.urlopen(base + "/health", timeout=30) as resp:
            assert json.loads(resp.read())["status"] == "ok"
        body = json.dumps({"prompt": "abc", "max_tokens": 5, "temperature": 0}).encode()
        req = urllib.request.Request(base + "/v1/completions", data=body, headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=60) as resp:
            out = json.loads(resp.read())
        assert out["usage"]["completion_tokens"] == 5
        body = json.dumps({"messages": [{"content": "abc"}], "model": "echo", "stream": True}).encode()
        req = urllib.request.Request(base + "/v1/chat/completions", data=body)
        with urllib.request.urlopen(req, timeout=60) as resp:
            text = resp.read().decode()
        assert text.rstrip().endswith("data: [DONE]")
        bad = urllib.request.Request(base + "/v1/completions", data=b"{not json")
        with pytest.raises(urllib.error.HTTPError) as ei:
            urllib.request.urlopen(bad, timeout=30)
        assert ei.value.code == 400
    finally:
        server.stop()


def test_http_server_keeps_json_connections_alive():
    """Two JSON requests over one HTTP/1.1 connection; an unknown route is a 404 and the server stops cleanly."""
    import http.client

    server = ServingServer(Router({"echo": EchoBackend()}, default_model="echo"), port=0)
    server.start()
    try:
        conn = http.client.HTTPConnection("127.0.0.1", server.port, timeout=30)
        for _ in range(2):
            conn.request("GET", "/v1/models")
            resp = conn.getresponse()
            assert resp.status == 200 and json.loads(resp.read())["data"][0]["id"] == "echo"
        conn.request("GET", "/nope")
        resp = conn.getresponse()
        assert resp.status == 404
        resp.read()
        conn.close()
    finally:
        server.stop()


def test_http_core_streams_pieces_and_reports_a_failing_producer():
    """The shared asyncio core: a streamed body arrives piece by piece and a producer that fails mid-stream
    ends with an error event; sized bodies keep the connection open; an oversized body is refused."""
    import http.client

    from rl_project_b200.serving.http import MAX_BODY_BYTES, AsyncHTTPServer

    def pieces(fail):
        yield "data: 1\n\n"
        yield "data: 2\n\n"
        if fail:
            raise RuntimeError("backend lost")

    def app(method, target, headers, body):
        if target.startswith("/stream"):
            return 200, "text/event-stream", pieces("fail" in target)
        return 200, "application/json", json.dumps({"echo": body.decode(), "target": target}).encode()

    srv = AsyncHTTPServer(app, port=0, on_bad_request=lambda s, m: json.dumps({"error": m}).encode())
    srv.start()
    try:
        conn = http.client.HTTPConnection("127.0.0.1", srv.port, timeout=30)
        conn.request("POST", "/x?y=1", body=b"abc")
        resp = conn.getresponse()
        assert resp.status == 200 and json.loads(resp.read()) == {"echo": "abc", "target": "/x?y=1"}
        conn.request("GET", "/stream")
        assert conn.getresponse().read().decode() == "data: 1\n\ndata: 2\n\n"
        conn.close()
        conn = http.client.HTTPConnection("127.0.0.1", srv.port, timeout=30)
        conn.request("GET", "/stream-fail")
        text = conn.getresponse().read().decode()
        assert text.startswith("data: 1\n\ndata: 2\n\n") and "backend lost" in text
        conn.close()
        conn = http.client.HTTPConnection("127.0.0.1", srv.port, timeout=30)
        conn.putrequest("POST", "/big")
        conn.putheader("Content-Length", str(MAX_BODY_BYTES + 1))
        conn.endheaders()
        resp = conn.getresponse()
        assert resp.status == 413 and "too large" in json.loads(resp.read())["error"]
        conn.close()
    finally:
        srv.stop()
