"""HTTP surface (OpenAI + Ollama) on the deterministic echo model, in-process.

Mirrors the reference's in-process router tests (crates/server/src/lib.rs
tests with tower::ServiceExt::oneshot): protocol shapes, streaming framing,
limits, 429 + Retry-After, request ids, cache headers, protocol-shaped
404/405, authentication, Ollama NDJSON.
"""
import json
import math

import pytest
from fastapi.testclient import TestClient

from bloom_b200.engine.pipeline import EchoPipeline
from bloom_b200.server.app import ServerSettings, create_app


class FakeEmbedder:
    def embed(self, texts, normalize=True, dimensions=None):
        out = []
        for t in texts:
            v = [float((hash(t) >> (4 * i)) % 17 - 8) + (1.0 if w in t else 0.0)
                 for i, w in enumerate(["cat", "dog", "sun", "car", "tea", "sky", "red", "big"])]
            if dimensions:
                v = v[:dimensions]
            n = math.sqrt(sum(x * x for x in v)) or 1.0
            out.append([x / n for x in v])
        return out


class EmbedPipeline(EchoPipeline):
    def __init__(self):
        super().__init__()
        self.cfg.arch = "bert"
        self.embedder = FakeEmbedder()

    @property
    def is_embedding(self):
        return True


@pytest.fixture(scope="module")
def client():
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", max_concurrent=4))
    with TestClient(app) as c:
        yield c


def test_health_ready_metrics(client):
    assert client.get("/health").json() == {"status": "ok"}
    r = client.get("/ready").json()
    assert r["object"] == "bloom.readiness" and r["protocol_version"] == 3
    assert r["minimum_ui_protocol_version"] == 3 and r["maximum_ui_protocol_version"] == 3
    m = client.get("/metrics")
    assert m.status_code == 200 and "bloom_requests_total" in m.text


def test_models_and_unknown_model(client):
    d = client.get("/v1/models").json()
    assert d["object"] == "list" and d["data"][0]["id"] == "echo"
    r = client.post("/v1/chat/completions", json={"model": "other", "messages": [{"role": "user", "content": "x"}]})
    assert r.status_code == 404 and r.json()["error"]["code"] == "model_not_found"


def test_chat_non_stream(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hello there"}]})
    assert r.status_code == 200
    d = r.json()
    assert d["object"] == "chat.completion"
    assert d["choices"][0]["message"] == {"role": "assistant", "content": "echo: hello there"}
    assert d["usage"]["completion_tokens"] > 0
    assert r.headers["cache-control"] == "no-store" and r.headers["x-request-id"]


def test_chat_stream_framing_and_usage(client):
    with client.stream("POST", "/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "a b c"}], "stream": True,
            "stream_options": {"include_usage": True}}) as r:
        lines = [l for l in r.iter_lines() if l]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant", "content": ""}
    text = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks if c["choices"])
    assert text == "echo: a b c"
    assert chunks[-1]["choices"] == [] and chunks[-1]["usage"]["completion_tokens"] > 0
    assert any(c["choices"] and c["choices"][0]["finish_reason"] for c in chunks)


def test_stop_sequence_never_leaks(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "one two three four"}],
                                                  "stop": ["three"]})
    d = r.json()
    assert d["choices"][0]["message"]["content"] == "echo: one two "
    assert d["choices"][0]["finish_reason"] == "stop"


def test_max_tokens_length(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "a b c d e f"}],
                                                  "max_tokens": 2})
    d = r.json()
    assert d["choices"][0]["finish_reason"] == "length"


@pytest.mark.parametrize("bad", [{"temperature": 5}, {"top_p": 0}, {"max_tokens": 0}, {"max_tokens": 40000},
                                 {"stop": ["a", "b", "c", "d", "e"]}, {"messages": []}])
def test_validation_errors(client, bad):
    body = {"messages": [{"role": "user", "content": "x"}]}
    body.update(bad)
    r = client.post("/v1/chat/completions", json=body)
    assert r.status_code == 400
    assert "message" in r.json()["error"]


def test_request_id_echo(client):
    r = client.get("/v1/models", headers={"x-request-id": "abc-123"})
    assert r.headers["x-request-id"] == "abc-123"


def test_protocol_shaped_404_405(client):
    r = client.get("/v1/nope")
    assert r.status_code == 404 and "error" in r.json() and isinstance(r.json()["error"], dict)
    r = client.get("/api/nope")
    assert r.status_code == 404 and isinstance(r.json()["error"], str)
    r = client.get("/v1/chat/completions")
    assert r.status_code == 405


def test_completions_and_responses(client):
    r = client.post("/v1/completions", json={"prompt": "hi you", "max_tokens": 10}).json()
    assert r["object"] == "text_completion" and r["choices"][0]["text"] == "echo: hi you"
    r = client.post("/v1/responses", json={"input": "ping", "instructions": "be brief"}).json()
    assert r["object"] == "response" and r["status"] == "completed"
    assert r["output"][0]["content"][0]["text"] == "echo: ping"
    got = client.get(f"/v1/responses/{r['id']}").json()
    assert got["id"] == r["id"]
    items = client.get(f"/v1/responses/{r['id']}/input_items").json()
    assert items["data"][-1]["content"][0]["text"] == "ping"
    assert client.get("/v1/responses/resp_missing").status_code == 404


def test_responses_stream_events(client):
    with client.stream("POST", "/v1/responses", json={"input": "x y", "stream": True}) as r:
        events = [l[7:] for l in r.iter_lines() if l.startswith("event: ")]
    assert events[0] == "response.created" and events[-1] == "response.completed"
    assert "response.output_text.delta" in events


def test_capacity_429():
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", max_concurrent=0))
    with TestClient(app) as c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}]})
        assert r.status_code == 429 and r.headers["retry-after"] == "1"


def test_api_key_auth():
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", api_keys=["s3cret"]))
    with TestClient(app) as c:
        r = c.get("/v1/models")
        assert r.status_code == 401 and "Bearer" in r.headers["www-authenticate"]
        assert c.get("/v1/models", headers={"Authorization": "Bearer s3cret"}).status_code == 200
        assert c.get("/health").status_code == 200


def test_ollama_surface(client):
    assert "version" in client.get("/api/version").json()
    assert client.get("/api/tags").json()["models"][0]["name"] == "echo"
    with client.stream("POST", "/api/chat", json={"model": "echo", "messages": [{"role": "user", "content": "q w"}]}) as r:
        rows = [json.loads(l) for l in r.iter_lines() if l]
    assert rows[-1]["done"] is True and rows[-1]["done_reason"] in ("stop", "length")
    assert "".join(x["message"]["content"] for x in rows) == "echo: q w"
    g = client.post("/api/generate", json={"model": "echo", "prompt": "z", "stream": False}).json()
    assert g["done"] and g["response"] == "echo: z"


def test_embeddings_and_rerank():
    app = create_app(EmbedPipeline(), ServerSettings(model_id="mini"))
    with TestClient(app) as c:
        d = c.post("/v1/embeddings", json={"input": ["the cat", "a dog"]}).json()
        assert d["object"] == "list" and len(d["data"]) == 2
        v = d["data"][0]["embedding"]
        assert abs(sum(x * x for x in v) - 1.0) < 1e-6
        d2 = c.post("/v1/embeddings", json={"input": "x", "dimensions": 4}).json()
        assert len(d2["data"][0]["embedding"]) == 4
        b = c.post("/v1/embeddings", json={"input": "x", "encoding_format": "base64"}).json()
        assert isinstance(b["data"][0]["embedding"], str)
        assert c.post("/v1/embeddings", json={"input": ["x"] * 257}).status_code == 400
        rr = c.post("/v1/rerank", json={"query": "cat", "documents": ["dog", "cat", "sun"], "top_n": 2}).json()
        assert len(rr["results"]) == 2
        scores = [x["relevance_score"] for x in rr["results"]]
        assert scores == sorted(scores, reverse=True)
        e = c.post("/api/embed", json={"model": "mini", "input": ["a", "b"]}).json()
        assert len(e["embeddings"]) == 2
        assert c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}]}).status_code == 400


def test_model_management(tmp_path):
    """Catalog list / preflight / switch / unload / remove on a models directory."""
    from bloom_b200.formats.gguf import GGML_Q8_0, write_decoder_gguf
    from bloom_b200.models.config import preset
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    write_decoder_gguf(str(tmp_path / "tiny.gguf"), cfg, random_weights(cfg, seed=0, std=0.08), GGML_Q8_0)
    (tmp_path / "broken").mkdir()
    (tmp_path / "spare.gguf").write_bytes((tmp_path / "tiny.gguf").read_bytes())
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", models_dir=str(tmp_path)))
    from bloom_b200.engine.pipeline import InferencePipeline

    app.state.model_loader = lambda path: InferencePipeline.load(path, device="cpu", context_size=256)
    with TestClient(app) as c:
        d = c.get("/v1/model-management/models").json()
        ids = {e["id"]: e for e in d["data"]}
        assert ids["tiny.gguf"]["valid"] and ids["tiny.gguf"]["primary_dtype"] == "Q8" and not ids["broken"]["valid"]
        pf = c.post("/v1/model-management/preflight", json={"model": "tiny.gguf", "context_size": 256}).json()
        assert pf["fits"] is True and pf["model"] == "tiny.gguf"
        assert c.post("/v1/model-management/preflight", json={"model": "nope"}).status_code == 404
        r = c.post("/v1/model-management/switch", json={"model": "tiny.gguf"})
        assert r.status_code == 200 and r.json()["model"] == "tiny.gguf"
        out = c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 3, "temperature": 0}).json()
        assert out["model"] == "tiny.gguf" and out["usage"]["completion_tokens"] >= 1
        assert c.delete("/v1/model-management/models/tiny.gguf?confirm=true").status_code == 409
        assert c.delete("/v1/model-management/models/spare.gguf").status_code == 400
        assert c.delete("/v1/model-management/models/spare.gguf?confirm=true").json()["status"] == "removed"
        assert not (tmp_path / "spare.gguf").exists()
        assert c.post("/v1/model-management/unload").json()["status"] == "unloaded"
        assert c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 3}).status_code == 503
        assert c.post("/api/pull", json={"model": "x"}).status_code == 501


def test_token_rate_limit(monkeypatch):
    monkeypatch.setenv("BLOOM_RATE_LIMIT", "1")
    monkeypatch.setenv("BLOOM_RATE_LIMIT_BURST", "100")
    monkeypatch.setenv("BLOOM_RATE_LIMIT_RATE", "1")
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo"))
    with TestClient(app) as c:
        ok = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 90})
        assert ok.status_code == 200
        r = c.post("/v1/completions", json={"prompt": "b", "max_tokens": 90})
        assert r.status_code == 429 and int(r.headers["retry-after"]) >= 1
        assert app.state.rate_limiter.throttled == 1


# ---------------------------------------------------------------- function tools
class ScriptedPipeline(EchoPipeline):
    """Streams a fixed text regardless of the prompt (the model's 'answer')."""

    answer = ""

    def run_stream(self, messages, params, raw: bool = False, stop=None, prompt_ids=None):
        self.last_prompt = messages
        self.last_params = params
        words = self.answer.split(" ")
        self.last_generated_tokens = len(words)
        for i, w in enumerate(words):
            yield w if i == 0 else " " + w


TOOLS = [{"type": "function", "function": {
    "name": "get_weather", "description": "Get weather.",
    "parameters": {"type": "object", "properties": {"city": {"type": "string"}}, "required": ["city"],
                   "additionalProperties": False}}}]


@pytest.fixture()
def scripted():
    pipe = ScriptedPipeline()
    app = create_app(pipe, ServerSettings(model_id="echo", max_concurrent=4))
    with TestClient(app) as c:
        yield c, pipe


def test_chat_tool_calls_non_stream_and_stream(scripted):
    c, pipe = scripted
    pipe.answer = '{"type": "function_calls", "calls": [{"name": "get_weather", "arguments": {"city": "Oslo"}}]}'
    body = {"model": "echo", "messages": [{"role": "user", "content": "weather in Oslo?"}], "tools": TOOLS,
            "max_tokens": 64}
    r = c.post("/v1/chat/completions", json=body)
    assert r.status_code == 200, r.text
    ch = r.json()["choices"][0]
    assert ch["finish_reason"] == "tool_calls" and ch["message"]["content"] is None
    call = ch["message"]["tool_calls"][0]
    assert call["type"] == "function" and call["function"]["name"] == "get_weather"
    assert json.loads(call["function"]["arguments"]) == {"city": "Oslo"}
    assert call["id"].startswith("call_")
    # the request ran constrained to the envelope, with the protocol in the prompt
    assert pipe.last_params.json_schema["properties"]["type"]["enum"] == ["message", "function_calls"]
    assert "get_weather" in pipe.last_prompt[-1]["content"]
    r = c.post("/v1/chat/completions", json=dict(body, stream=True))
    events = [json.loads(l[6:]) for l in r.text.splitlines() if l.startswith("data: {")]
    last = events[-1]["choices"][0]
    assert last["finish_reason"] == "tool_calls" and last["delta"]["tool_calls"][0]["index"] == 0
    assert r.text.rstrip().endswith("data: [DONE]")
    # a plain message through the same protocol
    pipe.answer = '{"type": "message", "content": "It is sunny."}'
    ch = c.post("/v1/chat/completions", json=body).json()["choices"][0]
    assert ch["finish_reason"] == "stop" and ch["message"]["content"] == "It is sunny."


def test_chat_tool_protocol_errors(scripted):
    c, pipe = scripted
    base = {"model": "echo", "messages": [{"role": "user", "content": "x"}]}
    r = c.post("/v1/chat/completions", json=dict(base, tools=[{"type": "function", "function": {"name": "a b"}}]))
    assert r.status_code == 400 and "ASCII" in r.json()["error"]["message"]
    r = c.post("/v1/chat/completions", json=dict(base, tool_choice="required"))
    assert r.status_code == 400
    pipe.answer = '{"type": "message", "content": "no"}'
    r = c.post("/v1/chat/completions", json=dict(base, tools=TOOLS, tool_choice="required"))
    assert r.status_code == 502 and "protocol" in r.json()["error"]["message"]
    # history: a tool call must be answered before the conversation continues
    call = {"id": "call_1", "type": "function", "function": {"name": "get_weather", "arguments": '{"city":"Oslo"}'}}
    msgs = [{"role": "user", "content": "w?"}, {"role": "assistant", "content": None, "tool_calls": [call]},
            {"role": "user", "content": "and?"}]
    r = c.post("/v1/chat/completions", json=dict(base, messages=msgs, tools=TOOLS))
    assert r.status_code == 400
    msgs[2] = {"role": "tool", "tool_call_id": "call_1", "content": "sunny, 21 C"}
    pipe.answer = '{"type": "message", "content": "Sunny."}'
    r = c.post("/v1/chat/completions", json=dict(base, messages=msgs, tools=TOOLS))
    assert r.status_code == 200 and r.json()["choices"][0]["message"]["content"] == "Sunny."
    assert any("untrusted" in m["content"] for m in pipe.last_prompt)


def test_response_format_schema_validation(scripted):
    c, pipe = scripted
    base = {"model": "echo", "messages": [{"role": "user", "content": "x"}]}
    bad = {"type": "json_schema", "json_schema": {"name": "s", "schema": {"type": "object", "properties": {
        "a": {"type": "string", "pattern": "x"}}}}}
    r = c.post("/v1/chat/completions", json=dict(base, response_format=bad))
    assert r.status_code == 400 and "pattern" in r.json()["error"]["message"]
    good = {"type": "json_schema", "json_schema": {"name": "s", "schema": {"type": "object", "properties": {
        "a": {"type": "string"}}, "required": ["a"]}}}
    pipe.answer = '{"a": "b"}'
    r = c.post("/v1/chat/completions", json=dict(base, response_format=good))
    assert r.status_code == 200 and json.loads(r.json()["choices"][0]["message"]["content"]) == {"a": "b"}
    assert pipe.last_params.json_schema == good["json_schema"]["schema"]


def test_responses_api_function_call(scripted):
    c, pipe = scripted
    pipe.answer = '{"type": "function_calls", "calls": [{"name": "get_weather", "arguments": {"city": "Rome"}}]}'
    flat = [dict(TOOLS[0]["function"], type="function")]
    r = c.post("/v1/responses", json={"model": "echo", "input": "weather?", "tools": flat})
    assert r.status_code == 200, r.text
    d = r.json()
    item = d["output"][0]
    assert item["type"] == "function_call" and item["name"] == "get_weather"
    assert json.loads(item["arguments"]) == {"city": "Rome"} and item["call_id"].startswith("call_")
    assert d["tools"][0]["name"] == "get_weather" and d["tool_choice"] == "auto"


def test_metrics_latency_memory_and_spans(client):
    for _ in range(2):
        client.post("/v1/chat/completions", json={"model": "echo", "messages": [{"role": "user", "content": "a b c"}]})
    text = client.get("/metrics").text
    for name in ("bloom_inter_token_latency_seconds_count", "bloom_request_latency_seconds", "bloom_uptime_seconds",
                 "bloom_process_resident_memory_bytes", "bloom_system_memory_total_bytes",
                 "bloom_memory_pressure_high", "bloom_requests_completed_total"):
        assert name in text, name
    obs = client.get("/v1/observability").json()
    assert obs["memory"]["rss_bytes"] > 0 and obs["memory"]["total_ram_bytes"] > 0
    assert "spans" in obs and obs["metrics"]["uptime_seconds"] >= 0


def test_tracing_spans_and_chrome_trace(tmp_path, monkeypatch):
    from bloom_b200.utils import tracing

    monkeypatch.setattr(tracing, "_TRACE_PATH", str(tmp_path / "t.json"))
    with tracing.span("unit.outer", k=1):
        with tracing.span("unit.inner"):
            pass
    st = tracing.stats()
    assert st["unit.outer"]["count"] >= 1 and st["unit.inner"]["seconds"] >= 0
    path = tracing.flush()
    ev = json.load(open(path))["traceEvents"]
    names = [e["name"] for e in ev]
    assert "unit.outer" in names and "unit.inner" in names
    outer = [e for e in ev if e["name"] == "unit.outer"][-1]
    assert outer["ph"] == "X" and outer["args"] == {"k": 1}


def test_memory_telemetry_snapshot():
    from bloom_b200.utils.telemetry import MemoryTelemetry

    s = MemoryTelemetry.snapshot([])
    assert s.rss_bytes > 0 and s.peak_rss_bytes >= s.rss_bytes and s.total_ram_bytes > s.rss_bytes
    assert 0.0 <= s.ram_utilization <= 1.0 and "RAM rss" in s.summary()
    assert s.to_dict()["high_pressure"] in (True, False)


def test_multimodal_stream_and_upload(client):
    import base64
    import sys
    import os

    sys.path.insert(0, os.path.dirname(__file__))
    import numpy as np
    from test_processor_vl import png_bytes

    img = np.random.default_rng(0).integers(0, 256, (12, 20, 3), dtype=np.uint8)
    png = png_bytes(img, 4)
    body = {"blocks": [{"Image": {"bytes": base64.b64encode(png).decode(), "mime": "image/png"}},
                       {"Text": "what is this"}], "params": {"max_tokens": 64}}
    r = client.post("/v1/multimodal/stream", json=body)
    ev = [json.loads(l[6:]) for l in r.text.splitlines() if l.startswith("data: ")]
    text = "".join(e["TextDelta"] for e in ev if isinstance(e, dict) and "TextDelta" in e)
    assert text == "echo: [image 20x12] what is this" and ev[-1] == "End"
    bad = client.post("/v1/multimodal/stream", json={"blocks": [{"Image": {"bytes": "AAAA", "mime": "image/jpeg"}},
                                                                {"Image": {"bytes": "AAAA", "mime": "x"}}]})
    assert bad.status_code == 400
    files = {"image": ("a.png", png, "image/png"), "prompt": (None, "hi")}
    r = client.post("/v1/multimodal/upload", files=files)
    ev = [json.loads(l[6:]) for l in r.text.splitlines() if l.startswith("data: ")]
    assert "".join(e["TextDelta"] for e in ev if isinstance(e, dict) and "TextDelta" in e) == \
        "echo: [image 20x12] hi"


def test_browser_origin_policy_and_preflight():
    """Reference: crates/server/src/lib.rs:12081-12240 (fail-closed origin guard aligned with CORS)."""
    from bloom_b200.server.app import origin_permitted

    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", cors_origins=["https://ui.example"]))
    with TestClient(app, base_url="http://127.0.0.1:3000") as c:
        ok = c.get("/health", headers={"origin": "https://ui.example"})
        assert ok.status_code == 200 and ok.headers["access-control-allow-origin"] == "https://ui.example"
        assert "x-request-id" in ok.headers["access-control-expose-headers"]
        same = c.get("/health", headers={"origin": "http://127.0.0.1:3000"})
        assert same.status_code == 200 and same.headers["access-control-allow-origin"] == "https://ui.example"
        assert c.get("/health").status_code == 200  # no Origin: not a browser
        for path, family in (("/v1/models", "openai"), ("/api/version", "ollama")):
            r = c.get(path, headers={"origin": "https://malicious.example"})
            assert r.status_code == 403 and r.headers["cache-control"] == "no-store"
            assert "x-request-id" in r.headers and "access-control-allow-origin" not in r.headers
            body = r.json()
            assert (body["error"]["type"] == "invalid_request_error") if family == "openai" else isinstance(
                body["error"], str)
        pre = c.options("/v1/models", headers={"origin": "https://malicious.example",
                                               "access-control-request-method": "GET"})
        assert pre.status_code == 403
        pre = c.options("/v1/chat/completions", headers={"origin": "https://ui.example",
                                                         "access-control-request-method": "POST",
                                                         "access-control-request-headers": "content-type"})
        assert pre.status_code == 204 and pre.headers["access-control-allow-origin"] == "https://ui.example"
    # DNS rebinding: a loopback listener refuses non-loopback page origins even when Host matches
    for origin in ("null", "http://attacker.example"):
        assert not origin_permitted([], True, [origin], "attacker.example")
    assert not origin_permitted(["https://ui.example"], True, ["https://ui.example", "https://x.example"], "h")
    assert origin_permitted(["*"], True, ["https://anything.example"], "127.0.0.1:3000")
    assert origin_permitted([], False, ["http://box.lan:8080"], "box.lan:8080")
    assert not origin_permitted([], False, ["https://box.lan:8080"], "box.lan:8080")  # same-origin is http only


def test_body_limit_and_concurrent_ndjson_streams(client):
    big = b"{" + b" " * (17 * 1024 * 1024) + b"}"
    r = client.post("/v1/chat/completions", content=big, headers={"content-type": "application/json"})
    assert r.status_code == 413 and r.json()["error"]["message"] == "request body too large"
    r = client.post("/api/chat", content=big, headers={"content-type": "application/json"})
    assert r.status_code == 413 and isinstance(r.json()["error"], str)

    import threading

    results, errors = {}, []
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", max_concurrent=8))
    cc = TestClient(app)
    cc.__enter__()

    def stream(i):
        try:
            lines = []
            with cc.stream("POST", "/api/generate", json={"model": "echo", "prompt": f"p{i} a b c"}) as s:
                assert s.headers["content-type"].startswith("application/x-ndjson")
                for line in s.iter_lines():
                    if line:
                        lines.append(json.loads(line))
            results[i] = lines
        except Exception as e:  # pragma: no cover - reported below
            errors.append(repr(e))

    ts = [threading.Thread(target=stream, args=(i,)) for i in range(6)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    cc.__exit__(None, None, None)
    assert not errors, errors
    assert len(results) == 6
    for i, lines in results.items():
        assert lines[-1]["done"] is True and all(not l["done"] for l in lines[:-1])
        text = "".join(l.get("response", "") for l in lines)
        assert f"p{i}" in text  # each stream carries its own request's output, none interleaved
