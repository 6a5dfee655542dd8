"""World-model loop (reference: crates/engine/src/world/mod.rs tests and the
/v1/world/step route): state cache eviction / TTL / compression, degradation
under thermal and power pressure, schema validation, chunk wire format."""
import json

import pytest
from fastapi.testclient import TestClient

from bloom_b200.engine import world as W


def st(i, n=128, t=1000):
    return W.WorldState(f"s{i}", i, t, [0.5] * (n // 4))


def test_state_cache_budget_priority_ttl_compress():
    c = W.StateCache(W.CacheConfig(max_bytes=200, max_entries=2, auto_compress=False))
    c.insert(st(0, 100), "Low")
    c.insert(st(1, 100), "High")
    c.insert(st(2, 100), "Normal")  # evicts the Low entry
    assert set(c.states) == {"s1", "s2"} and c.total_bytes == 200
    with pytest.raises(W.WorldError):
        W.StateCache(W.CacheConfig(max_bytes=50)).insert(st(0, 100))
    c = W.StateCache(W.CacheConfig(default_ttl_ms=500, compress_after_ms=100))
    c.insert(st(0, 128, t=1000))
    assert c.compress_old(1200) == 1 and c.total_bytes == 64
    assert c.expire(1400) == [] and c.expire(1600) == ["s0"] and c.total_bytes == 0


def test_constraints_from_thermal_power():
    assert not W.Constraints.from_thermal_power("Nominal", "PluggedIn").degraded
    s = W.Constraints.from_thermal_power("Serious", "PluggedIn")
    assert s.observation_skip_ratio == 2 and s.effective_horizon(10) == 4
    c = W.Constraints.from_thermal_power("Critical", "Battery")
    assert c.effective_horizon(10) == 1 and c.suggest_smaller_model
    assert W.Constraints.from_thermal_power("Nominal", "Battery").effective_horizon(10) == 2
    assert [s.should_skip(i) for i in range(4)] == [False, True, False, True]


def test_mock_loop_steps_and_validation():
    loop = W.WorldModelLoop(W.MockWorldModel(), W.MockPolicy("robot_velocity", 2))
    ch = loop.step([W.Observation.parse({"Scalar": {"name": "speed", "value": 1.5}})], 3)
    assert ch[0] == {"StateDelta": {"from_state_id": "init", "to_state_id": "state-0", "latent_update": None}}
    assert [c["PredictedState"]["horizon_step"] for c in ch[1:4]] == [1, 2, 3]
    assert ch[4]["Action"] == {"action_space": "robot_velocity", "values": [1.0, 1.0]} and ch[-1] == "End"
    ch = loop.step([], 1)
    assert ch[0]["StateDelta"]["from_state_id"] == "state-0"
    loop.state_schema = {"scalar_ranges": {"speed": [0, 1]}, "allow_text": False}
    with pytest.raises(W.WorldError, match="out of range"):
        loop.step([W.Observation.parse({"Scalar": {"name": "speed", "value": 2.0}})])
    with pytest.raises(W.WorldError, match="Text"):
        loop.step([W.Observation.parse({"Text": "hi"})])
    loop.state_schema = None
    loop.action_schema = {"action_dimensions": {"robot_velocity": 3}}
    with pytest.raises(W.WorldError, match="expected dimension 3"):
        loop.step([])
    for bad in ({"Foo": 1}, {"Scalar": {"name": 1, "value": 2}}, {"Image": {"bytes": [300], "mime": "x"}}):
        with pytest.raises(W.WorldError):
            W.Observation.parse(bad)


def test_latent_loop_is_deterministic_and_degrades():
    obs = [W.Observation.parse({"Scalar": {"name": "x", "value": 3.0}}), W.Observation.parse({"Text": "door open"}),
           W.Observation.parse({"AudioPcm": {"samples": [0.1, -0.2, 0.3], "sample_rate": 16000}})]
    a = W.WorldModelLoop(W.LatentWorldModel(dim=64, device="cpu"), W.LinearPolicy(64, "arm", 3))
    b = W.WorldModelLoop(W.LatentWorldModel(dim=64, device="cpu"), W.LinearPolicy(64, "arm", 3))
    ca, cb = a.step(obs, 4), b.step(obs, 4)
    assert ca[:-1][:5] == cb[:-1][:5]  # same seed -> same states, futures and action
    acts = [c["Action"] for c in ca if isinstance(c, dict) and "Action" in c][0]
    assert acts["action_space"] == "arm" and len(acts["values"]) == 3 and all(-1 <= v <= 1 for v in acts["values"])
    conf = [c["PredictedState"]["confidence"] for c in ca if isinstance(c, dict) and "PredictedState" in c]
    assert len(conf) == 4 and all(x > y for x, y in zip(conf, conf[1:]))
    a.set_environment("Critical", "PluggedIn")  # horizon 1, observe one step in three
    ch = a.step(obs, 4)
    assert sum(1 for c in ch if isinstance(c, dict) and "PredictedState" in c) == 1


def test_world_step_route():
    from bloom_b200.engine.pipeline import EchoPipeline
    from bloom_b200.server.app import ServerSettings, create_app

    with TestClient(create_app(EchoPipeline(), ServerSettings(model_id="echo"))) as c:
        body = {"observations": [{"Scalar": {"name": "v", "value": 1.0}}], "horizon": 2, "engine": "mock"}
        r = c.post("/v1/world/step", json=body).json()
        assert r[0]["StateDelta"]["to_state_id"] == "state-0" and r[-1] == "End"
        r = c.post("/v1/world/step", json=dict(body, session="s")).json()
        r = c.post("/v1/world/step", json=dict(body, session="s")).json()
        assert r[0]["StateDelta"]["from_state_id"] == "state-0"  # the session kept its state
        s = c.post("/v1/world/step", json=dict(body, stream=True))
        events = [json.loads(l[6:]) for l in s.text.splitlines() if l.startswith("data: ")]
        assert events[-1] == "End" and "Action" in events[-3]
        bad = c.post("/v1/world/step", json={"observations": [{"Nope": 1}]})
        assert bad.status_code == 400
        r = c.post("/v1/world/step", json={"observations": [{"Text": "hello"}], "horizon": 1}).json()
        assert r[0]["StateDelta"]["to_state_id"].startswith("latent-0-")
