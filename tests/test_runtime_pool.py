"""Multi-model residency: runtime pool, aggregate memory permits, Ollama
keep_alive (reference: crates/server/src/runtime_pool.rs tests,
runtime_memory.rs, ollama.rs keep_alive parsing and residency)."""
import time

import pytest
from fastapi.testclient import TestClient

from bloom_b200.server.runtime_pool import (INDEFINITE, Footprint, KeepAliveError, MemoryBudget, MemoryError_,
                                            RuntimeEntry, RuntimePool, parse_keep_alive)


class FakeRuntime:
    def __init__(self):
        self.down = False
        self.in_flight = 0

    def shutdown(self):
        self.down = True


def entry(key, fp=None, budget=None):
    return RuntimeEntry(key, f"/m/{key}", object(), FakeRuntime(), budget.reserve(fp) if budget else None)


def test_keep_alive_parsing():
    assert parse_keep_alive(None) == 300.0
    assert parse_keep_alive(0) == 0.0 and parse_keep_alive("0") == 0.0
    assert parse_keep_alive(-1) == INDEFINITE and parse_keep_alive("-5m") == INDEFINITE
    assert parse_keep_alive("5m") == 300.0 and parse_keep_alive("1h30m") == 5400.0
    assert parse_keep_alive("250ms") == pytest.approx(0.25) and parse_keep_alive("1.5s") == 1.5
    assert parse_keep_alive(42) == 42.0 and parse_keep_alive("42") == 42.0
    for bad in ("", "5x", "m5", True, [1], "1h 5m", "400d", 10 ** 9, float("nan")):
        with pytest.raises(KeepAliveError):
            parse_keep_alive(bad)


def test_pool_capacity_evicts_oldest_non_default():
    p = RuntimePool(capacity=3)
    a, b, c, d = (entry(k) for k in "abcd")
    assert p.publish(a, make_default=True) == []
    p.publish(b)
    p.publish(c)
    retired = p.publish(d)
    assert retired == [b] and p.default_key == "a"  # the default stays pinned
    assert [e.key for e in p.entries()] == ["a", "c", "d"]
    e2 = entry("c")
    assert p.publish(e2) == [c] and p.get("c") is e2  # same key: the old generation retires
    one = RuntimePool(capacity=1)
    one.publish(a, make_default=True)
    assert one.publish(b) == [a] and one.default_key == "b"
    assert p.select(None) is a and p.select("d") is d and p.select("zzz") is None


def test_memory_budget_permits():
    b = MemoryBudget(host_limit_bytes=100, device_limit_bytes=1000)
    p1 = b.reserve(Footprint(40, 600))
    ok, why, snap = b.evaluate(Footprint(0, 500))
    assert not ok and "device memory budget" in why and snap["device_used_bytes"] == 600
    with pytest.raises(MemoryError_):
        b.reserve(Footprint(70, 0))
    p2 = b.reserve(Footprint(60, 400))
    assert b.snapshot()["generations"] == 2
    p1.release()
    p1.release()  # idempotent
    assert b.snapshot() == {"host_limit_bytes": 100, "host_used_bytes": 60, "device_limit_bytes": 1000,
                            "device_used_bytes": 400, "generations": 1}
    p2.resize(Footprint(10, 900))
    assert b.snapshot()["device_used_bytes"] == 900
    with pytest.raises(MemoryError_):
        p2.resize(Footprint(10, 1100))
    with pytest.raises(MemoryError_):
        b.reserve(Footprint(0, 50), available=Footprint(0, 10))


def test_evict_for_frees_idle_lru_entries():
    b = MemoryBudget(1 << 40, 1000)
    p = RuntimePool(capacity=4)
    a, x, y = entry("a", Footprint(0, 300), b), entry("x", Footprint(0, 300), b), entry("y", Footprint(0, 300), b)
    p.publish(a, make_default=True)
    p.publish(x)
    p.publish(y)
    p.touch("y")
    x.last_used = time.time() - 100
    y.runtime.in_flight = 1  # busy: never evicted
    gone = p.evict_for(b, Footprint(0, 300))
    assert [g.key for g in gone] == ["x"] and x.runtime.down and b.snapshot()["device_used_bytes"] == 600
    assert p.evict_for(b, Footprint(0, 900)) == []  # only the default and a busy entry are left


def test_keep_alive_deadlines():
    p = RuntimePool(capacity=2)
    a, b = entry("a"), entry("b")
    p.publish(a, make_default=True)
    p.publish(b)
    p.touch("b", 0.5)
    assert b.expires_at is not None and p.expired(time.time()) == []
    assert p.expired(time.time() + 1.0) == ["b"]
    p.touch("b", INDEFINITE)
    assert b.expires_at is None and p.expired(time.time() + 1e6) == []


# ---------------------------------------------------------------- HTTP
def _server(tmp_path, capacity=2, device_limit=0, host_limit=0):
    from bloom_b200.engine.pipeline import EchoPipeline
    from bloom_b200.formats.gguf import GGML_Q8_0, write_decoder_gguf
    from bloom_b200.models.config import preset
    from bloom_b200.models.reference import random_weights
    from bloom_b200.server.app import ServerSettings, create_app

    cfg = preset("tiny-llama")
    write_decoder_gguf(str(tmp_path / "m1.gguf"), cfg, random_weights(cfg, seed=0, std=0.08), GGML_Q8_0)
    (tmp_path / "m2.gguf").write_bytes((tmp_path / "m1.gguf").read_bytes())
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", models_dir=str(tmp_path), pool_capacity=capacity,
                                                    memory_host_limit=host_limit, memory_device_limit=device_limit))

    class Named(EchoPipeline):
        def __init__(self, path):
            super().__init__()
            self.path = path

        def run_stream(self, messages, params, raw=False, stop=None, prompt_ids=None):
            yield "from " + self.path.rsplit("/", 1)[-1]

    app.state.model_loader = lambda path: Named(path)
    return app


def test_http_residency_routes_requests_by_model(tmp_path):
    with TestClient(_server(tmp_path)) as c:
        r = c.post("/v1/model-management/load", json={"model": "m1.gguf"})
        assert r.status_code == 200 and r.json()["resident"] == ["echo", "m1.gguf"]
        out = c.post("/v1/chat/completions", json={"model": "m1.gguf", "messages": [{"role": "user", "content": "x"}]})
        assert out.json()["model"] == "m1.gguf" and out.json()["choices"][0]["message"]["content"] == "from m1.gguf"
        out = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}]}).json()
        assert out["model"] == "echo" and out["choices"][0]["message"]["content"].startswith("echo:")
        c.post("/v1/model-management/load", json={"model": "m2.gguf"})  # capacity 2: m1 (oldest non-default) goes
        res = c.get("/v1/model-management/residency").json()
        assert [m["model"] for m in res["models"]] == ["echo", "m2.gguf"] and res["default"] == "echo"
        assert res["memory_budget"]["generations"] == 1
        assert c.post("/v1/chat/completions", json={"model": "m1.gguf",
                                                    "messages": [{"role": "user", "content": "x"}]}).status_code == 404
        assert c.post("/v1/model-management/unload", json={"model": "m2.gguf"}).json()["status"] == "unloaded"
        assert c.get("/v1/model-management/residency").json()["memory_budget"]["generations"] == 0


def test_http_memory_budget_refuses_and_evicts(tmp_path):
    with TestClient(_server(tmp_path, capacity=4, device_limit=1, host_limit=1)) as c:
        r = c.post("/v1/model-management/load", json={"model": "m1.gguf"})
        assert r.status_code == 507 and "memory budget" in r.json()["error"]["message"]


def test_ollama_keep_alive_load_unload_and_expiry(tmp_path):
    with TestClient(_server(tmp_path, capacity=3)) as c:
        # generate naming a catalog model loads it on demand, with a short keep_alive
        r = c.post("/api/generate", json={"model": "m1.gguf", "prompt": "hi", "stream": False, "keep_alive": "300ms"})
        assert r.status_code == 200 and r.json()["response"] == "from m1.gguf"
        ps = c.get("/api/ps").json()["models"]
        assert {m["name"] for m in ps} == {"echo", "m1.gguf"}
        time.sleep(1.0)
        assert {m["name"] for m in c.get("/api/ps").json()["models"]} == {"echo"}
        # an empty request loads; keep_alive 0 unloads
        r = c.post("/api/generate", json={"model": "m2.gguf", "keep_alive": -1})
        assert r.json()["done_reason"] == "load"
        assert "m2.gguf" in {m["name"] for m in c.get("/api/ps").json()["models"]}
        r = c.post("/api/chat", json={"model": "m2.gguf", "keep_alive": 0})
        assert r.json()["done_reason"] == "unload"
        assert "m2.gguf" not in {m["name"] for m in c.get("/api/ps").json()["models"]}
        assert c.post("/api/generate", json={"model": "m1.gguf", "keep_alive": "5x"}).status_code == 400


def test_residency_reports_ledger(tmp_path):
    with TestClient(_server(tmp_path)) as c:
        c.post("/v1/model-management/load", json={"model": "m1.gguf"})
        led = c.get("/v1/model-management/residency").json()["ledger"]
        assert sum(v["used_bytes"] for v in led.values()) > 0
        c.post("/v1/model-management/unload", json={"model": "m1.gguf"})
        led = c.get("/v1/model-management/residency").json()["ledger"]
        assert sum(v["used_bytes"] for v in led.values()) == 0


def test_segment_admission_order():
    """Waiting requests are admitted by weighted fair queueing over request
    classes (foreground 4 : realtime 3 : background 2 : maintenance 1) and
    reach the engine with the class's priority."""
    import asyncio

    from bloom_b200.server.runtime import ServingRuntime

    class Eng:
        def __init__(self):
            self.added, self.live, self.requests = [], {}, {}
            self.n = 0

        def add_request(self, prompt, params, priority=0):
            self.n += 1
            self.added.append((prompt[0], priority))
            return self.n

        def abort(self, rid):
            pass

        def has_unfinished(self):
            return False

        def step(self):
            return []

    class Pipe:
        pass

    p = Pipe()
    p.llm = Eng()

    async def go():
        rt = ServingRuntime(p, "m", 64, admit_per_step=4)
        rt._stop.set()  # hold the loop: submit everything first
        rt._thread.join()
        subs = [rt.submit([100 + i], None, segment=2) for i in range(4)] + \
               [rt.submit([200 + i], None, segment=0) for i in range(4)]
        rt._stop.clear()
        import threading

        rt._thread = threading.Thread(target=rt._loop, daemon=True)
        rt._thread.start()
        await asyncio.sleep(0.3)
        rt.shutdown()
        return p.llm.added

    added = asyncio.run(go())
    assert len(added) == 8
    first = added[:4]  # one batch of 4: a weighted pass, foreground weight 4 > background 2
    assert sum(1 for t, _ in first if t >= 200) >= 2
    assert {pr for t, pr in added if t >= 200} == {3} and {pr for t, pr in added if t < 200} == {1}
