"""World-model loop: observation -> state -> predicted futures -> action.

A closed loop over a world model (`observe`: fold new observations into a
latent state; `predict`: roll the state forward `horizon` steps) and a
policy (`decide`: state, optionally with futures -> action), with a bounded
cache of past states and adaptive degradation under thermal / power
pressure (skip observations, shorten the horizon, suggest a smaller model).
Every step yields OutputChunk values in the engine's wire form (externally
tagged JSON): StateDelta, PredictedState per horizon step, Action, Metrics,
End.  Observations and actions are checked against optional schemas.

Engines
  LatentWorldModel / LinearPolicy   a latent dynamics model on the GPU: the
      observation features (scalars hashed into slots, text byte statistics,
      tensor / audio / image summaries) and the previous latent go through
      this repository's GEMM kernel (bf16, tanh), futures roll the latent
      forward, the policy reads an action vector out of the latent.  Weights
      are seeded random (no world-model checkpoint format exists to load).
  MockWorldModel / MockPolicy       the reference's deterministic test pair.

Reference: crates/engine/src/world/mod.rs:27-760 (WorldModelEngine,
PolicyEngine, StateCacheManager, WorldModelConstraints, WorldModelLoop,
mocks), crates/core/src/world.rs (types), server route /v1/world/step
(crates/server/src/handlers.rs:5114-5200).
"""
from __future__ import annotations

import base64
import math
import struct
import time
import zlib
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

THERMAL = ("Nominal", "Fair", "Serious", "Critical")
POWER = ("Battery", "PluggedIn")
PRIORITY = {"Low": 0, "Normal": 1, "High": 2, "Critical": 3}


class WorldError(ValueError):
    pass


def _now_ms() -> int:
    return int(time.time() * 1000)


# ---------------------------------------------------------------- observations
@dataclass
class Observation:
    kind: str  # Text | Image | AudioPcm | Tensor | Scalar
    value: Any

    @staticmethod
    def parse(o: Any) -> "Observation":
        """Externally tagged JSON: {"Text": "..."}, {"Scalar": {"name", "value"}},
        {"Image": {"bytes", "mime"}}, {"AudioPcm": {"samples", "sample_rate"}},
        {"Tensor": {"dtype", "shape", "bytes"}} (bytes as a list or base64)."""
        if not isinstance(o, dict) or len(o) != 1:
            raise WorldError("each observation must be an object with exactly one of Text, Image, AudioPcm, "
                             "Tensor, Scalar")
        kind, v = next(iter(o.items()))
        if kind == "Text":
            if not isinstance(v, str):
                raise WorldError("Text observation must be a string")
        elif kind == "Scalar":
            if not isinstance(v, dict) or not isinstance(v.get("name"), str) or \
                    not isinstance(v.get("value"), (int, float)) or isinstance(v.get("value"), bool):
                raise WorldError("Scalar observation needs a string name and a numeric value")
        elif kind == "Image":
            if not isinstance(v, dict) or not isinstance(v.get("mime"), str):
                raise WorldError("Image observation needs bytes and a mime type")
            v = dict(v, bytes=_bytes(v.get("bytes")))
        elif kind == "AudioPcm":
            if not isinstance(v, dict) or not isinstance(v.get("samples"), list):
                raise WorldError("AudioPcm observation needs samples and a sample_rate")
        elif kind == "Tensor":
            if not isinstance(v, dict) or not isinstance(v.get("shape"), list):
                raise WorldError("Tensor observation needs dtype, shape and bytes")
            v = dict(v, bytes=_bytes(v.get("bytes")))
        else:
            raise WorldError(f"unknown observation kind {kind!r}")
        return Observation(kind, v)


def _bytes(b: Any) -> bytes:
    if isinstance(b, str):
        return base64.b64decode(b)
    if isinstance(b, list) and all(isinstance(x, int) and 0 <= x < 256 for x in b):
        return bytes(b)
    raise WorldError("bytes must be a list of 0..255 or a base64 string")


@dataclass
class WorldState:
    state_id: str
    step: int
    timestamp_ms: int
    latent: Optional[List[float]] = None
    observations: List[Observation] = field(default_factory=list)

    @property
    def latent_bytes(self) -> int:
        return 4 * len(self.latent or [])


@dataclass
class Future:
    state_id: str
    confidence: float
    horizon_step: int
    latent: Optional[List[float]] = None


@dataclass
class Action:
    action_space: str
    values: List[float]
    metadata: Optional[str] = None


# ---------------------------------------------------------------- state cache
@dataclass
class CacheConfig:
    max_bytes: int = 256 * 1024 * 1024
    max_entries: int = 64
    default_ttl_ms: int = 0
    auto_compress: bool = True
    compress_after_ms: int = 60_000


class StateCache:
    """Cached world states: eviction of the lowest priority, least recently
    used entry when a byte or entry budget is hit; TTL expiry; entries older
    than compress_after_ms are compressed (their latent is stored as bf16,
    halving its bytes)."""

    def __init__(self, cfg: Optional[CacheConfig] = None):
        self.cfg = cfg or CacheConfig()
        self.entries: Dict[str, Dict] = {}
        self.states: Dict[str, WorldState] = {}
        self.total_bytes = 0

    def insert(self, st: WorldState, priority: str = "Normal") -> None:
        size = st.latent_bytes
        while self.total_bytes + size > self.cfg.max_bytes or len(self.entries) >= self.cfg.max_entries:
            if not self._evict_one():
                raise WorldError(f"state cache full ({self.total_bytes} bytes / {self.cfg.max_bytes} max, "
                                 f"{len(self.entries)} entries / {self.cfg.max_entries} max); cannot evict")
        self.entries[st.state_id] = {"size": size, "created": st.timestamp_ms, "last_access": st.timestamp_ms,
                                     "access_count": 0, "compressed": False, "priority": PRIORITY[priority],
                                     "ttl": self.cfg.default_ttl_ms}
        self.states[st.state_id] = st
        self.total_bytes += size

    def get(self, state_id: str) -> Optional[WorldState]:
        e = self.entries.get(state_id)
        if e is not None:
            e["last_access"] = _now_ms()
            e["access_count"] += 1
        return self.states.get(state_id)

    def remove(self, state_id: str) -> bool:
        e = self.entries.pop(state_id, None)
        if e is None:
            return False
        self.total_bytes -= e["size"]
        self.states.pop(state_id, None)
        return True

    def expire(self, now_ms: int) -> List[str]:
        gone = [k for k, e in self.entries.items() if e["ttl"] > 0 and now_ms - e["created"] > e["ttl"]]
        for k in gone:
            self.remove(k)
        return gone

    def compress_old(self, now_ms: int) -> int:
        if not self.cfg.auto_compress:
            return 0
        n = 0
        for k, e in self.entries.items():
            if not e["compressed"] and now_ms - e["created"] > self.cfg.compress_after_ms:
                st = self.states[k]
                if st.latent:  # keep the latent at bf16 precision
                    st.latent = [_bf16(x) for x in st.latent]
                saved = e["size"] // 2
                e["size"] -= saved
                e["compressed"] = True
                self.total_bytes -= saved
                n += 1
        return n

    def latest(self) -> Optional[WorldState]:
        return max(self.states.values(), key=lambda s: s.step, default=None)

    def _evict_one(self) -> bool:
        if not self.entries:
            return False
        victim = min(self.entries.items(), key=lambda kv: (kv[1]["priority"], kv[1]["last_access"]))[0]
        return self.remove(victim)


def _bf16(x: float) -> float:
    b = struct.unpack("<I", struct.pack("<f", x))[0]
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000  # round to nearest even
    return struct.unpack("<f", struct.pack("<I", b))[0]


# ---------------------------------------------------------------- constraints and schemas
@dataclass
class Constraints:
    thermal_state: str = "Nominal"
    power_state: str = "PluggedIn"
    observation_skip_ratio: int = 0
    max_degraded_horizon: int = 1 << 31
    suggest_smaller_model: bool = False

    @staticmethod
    def from_thermal_power(thermal: str, power: str) -> "Constraints":
        if thermal not in THERMAL or power not in POWER:
            raise WorldError(f"thermal_state must be one of {THERMAL}, power_state one of {POWER}")
        skip, horizon, smaller = {"Nominal": (0, 1 << 31, False), "Fair": (0, 1 << 31, False),
                                  "Serious": (2, 4, False), "Critical": (3, 1, True)}[thermal]
        if power == "Battery":
            horizon = min(horizon, 2)
        return Constraints(thermal, power, skip, horizon, smaller)

    def effective_horizon(self, requested: int) -> int:
        return min(int(requested), self.max_degraded_horizon)

    def should_skip(self, step: int) -> bool:
        return self.observation_skip_ratio > 0 and step % self.observation_skip_ratio != 0

    @property
    def degraded(self) -> bool:
        return self.observation_skip_ratio > 0 or self.max_degraded_horizon < (1 << 31) or \
            self.power_state == "Battery"


def validate_observation(obs: Observation, schema: Optional[Dict]) -> None:
    if not schema:
        return
    if obs.kind == "Text" and not schema.get("allow_text", True):
        raise WorldError("Text observations are not allowed by schema")
    if obs.kind == "AudioPcm" and not schema.get("allow_audio", True):
        raise WorldError("Audio observations are not allowed by schema")
    if obs.kind == "Image":
        mimes = schema.get("allowed_image_mimes") or []
        if mimes and obs.value["mime"] not in mimes:
            raise WorldError(f"Image MIME type '{obs.value['mime']}' is not allowed by schema")
    if obs.kind == "Tensor":
        shapes = schema.get("tensor_shapes") or []
        if shapes and list(obs.value["shape"]) not in [list(s) for s in shapes]:
            raise WorldError(f"Tensor shape {obs.value['shape']} is not allowed by schema")
    if obs.kind == "Scalar":
        rng = (schema.get("scalar_ranges") or {}).get(obs.value["name"])
        if rng is not None and not rng[0] <= obs.value["value"] <= rng[1]:
            raise WorldError(f"Scalar observation '{obs.value['name']}' value {obs.value['value']} is out of range "
                             f"[{rng[0]}, {rng[1]}]")


def validate_action(a: Action, schema: Optional[Dict]) -> None:
    if not schema:
        return
    spaces = schema.get("allowed_action_spaces") or []
    if spaces and a.action_space not in spaces:
        raise WorldError(f"Action space '{a.action_space}' is not allowed by schema")
    dim = (schema.get("action_dimensions") or {}).get(a.action_space)
    if dim is not None and len(a.values) != dim:
        raise WorldError(f"Action space '{a.action_space}' expected dimension {dim}, got {len(a.values)}")
    rng = schema.get("value_range")
    if rng is not None and any(not rng[0] <= v <= rng[1] for v in a.values):
        raise WorldError(f"Action values are outside the range [{rng[0]}, {rng[1]}]")


# ---------------------------------------------------------------- engines
class MockWorldModel:
    """Deterministic transitions: state-N from state-(N-1), futures with confidence 1/h."""

    name = "mock-world-model"

    def observe(self, cur: Optional[WorldState], obs: List[Observation], horizon: int) -> Tuple[WorldState, List[Future]]:
        step = cur.step + 1 if cur else 0
        st = WorldState(f"state-{step}", step, _now_ms(), None, obs)
        return st, self.predict(st, horizon)

    def predict(self, st: WorldState, horizon: int) -> List[Future]:
        return [Future(f"{st.state_id}-pred-{h}", 1.0 / h, h) for h in range(1, horizon + 1)]


class MockPolicy:
    name = "mock-policy"

    def __init__(self, action_space: str = "robot_velocity", dim: int = 2):
        self.space, self.dim = action_space, dim

    def decide(self, st: WorldState, futures: List[Future]) -> Action:
        base = st.step * 0.1
        if not futures:
            return Action(self.space, [base] * self.dim, f"step_{st.step}")
        best = max(f.confidence for f in futures)
        return Action(self.space, [base + best] * self.dim, f"step_{st.step}_with_future")


FEATURES = 64


def observation_features(obs: List[Observation]) -> List[float]:
    """A fixed-size feature vector: each observation adds its summary to
    slots chosen by a CRC of its name / kind."""
    f = [0.0] * FEATURES

    def put(key: str, vals: List[float]) -> None:
        h = zlib.crc32(key.encode())
        for i, v in enumerate(vals):
            f[(h + i) % FEATURES] += float(v)

    for o in obs:
        if o.kind == "Scalar":
            put("scalar:" + o.value["name"], [math.tanh(float(o.value["value"]) / 10.0)])
        elif o.kind == "Text":
            b = o.value.encode()
            put("text", [len(b) / 256.0, sum(b) / (255.0 * max(1, len(b))), b.count(b" ") / max(1, len(b))])
        elif o.kind == "AudioPcm":
            s = [float(x) for x in o.value["samples"]] or [0.0]
            put("audio", [math.sqrt(sum(x * x for x in s) / len(s)), max(abs(x) for x in s)])
        elif o.kind in ("Tensor", "Image"):
            b = o.value["bytes"] or b"\0"
            put(o.kind.lower(), [len(b) / 65536.0, sum(b) / (255.0 * len(b))])
    return f


class LatentWorldModel:
    """latent' = tanh(W_s latent + W_o features); futures roll
    latent_{h+1} = tanh(W_s latent_h), confidence 0.9^h scaled by how much
    the latent still moves.  The GEMMs run on this repository's kernel when
    a GPU is present (CPU fp32 otherwise)."""

    name = "latent-world-model"

    def __init__(self, dim: int = 256, seed: int = 0, device: Optional[str] = None):
        import torch

        g = torch.Generator().manual_seed(seed)
        self.dim = dim
        self.device = torch.device(device) if device else (
            torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu"))
        ws = torch.randn(dim, dim, generator=g) * (0.9 / math.sqrt(dim))
        wo = torch.randn(dim, FEATURES, generator=g) * (1.0 / math.sqrt(FEATURES))
        self.w = torch.cat([ws, wo], 1)  # [dim, dim + FEATURES]: one GEMM per step
        if self.device.type == "cuda":
            self.w = self.w.to(self.device, torch.bfloat16).contiguous()

    def _step(self, latent, feats):
        import torch

        x = torch.tensor(list(latent) + list(feats), dtype=torch.float32).view(1, -1)
        if self.device.type == "cuda":
            from .. import ops

            y = ops.gemm(x.to(self.device, torch.bfloat16), self.w).float()
        else:
            y = x @ self.w.t()
        return torch.tanh(y).view(-1).cpu().tolist()

    def observe(self, cur: Optional[WorldState], obs: List[Observation], horizon: int) -> Tuple[WorldState, List[Future]]:
        prev = cur.latent if cur and cur.latent else [0.0] * self.dim
        lat = self._step(prev, observation_features(obs))
        step = cur.step + 1 if cur else 0
        st = WorldState(f"latent-{step}-{zlib.crc32(struct.pack(f'<{len(lat)}f', *lat)) & 0xFFFFFFFF:08x}", step,
                        _now_ms(), lat, obs)
        return st, self.predict(st, horizon)

    def predict(self, st: WorldState, horizon: int) -> List[Future]:
        out, lat = [], st.latent or [0.0] * self.dim
        zero = [0.0] * FEATURES
        for h in range(1, horizon + 1):
            nxt = self._step(lat, zero)
            move = math.sqrt(sum((a - b) ** 2 for a, b in zip(nxt, lat)) / self.dim)
            out.append(Future(f"{st.state_id}-pred-{h}", round((0.9 ** h) / (1.0 + move), 6), h, nxt))
            lat = nxt
        return out


class LinearPolicy:
    """action = tanh(W_a mean(latent, most confident future latent))[:dim]."""

    name = "linear-policy"

    def __init__(self, latent_dim: int = 256, action_space: str = "robot_velocity", dim: int = 2, seed: int = 1):
        import torch

        g = torch.Generator().manual_seed(seed)
        self.space, self.dim = action_space, dim
        self.w = torch.randn(dim, latent_dim, generator=g) * (1.0 / math.sqrt(latent_dim))

    def decide(self, st: WorldState, futures: List[Future]) -> Action:
        import torch

        lat = torch.tensor(st.latent or [0.0] * self.w.shape[1])
        best = max(futures, key=lambda f: f.confidence, default=None)
        if best is not None and best.latent is not None:
            lat = 0.5 * (lat + torch.tensor(best.latent))
        vals = torch.tanh(self.w @ lat).tolist()
        return Action(self.space, [round(v, 6) for v in vals], f"step_{st.step}")


# ---------------------------------------------------------------- loop
class WorldModelLoop:
    def __init__(self, world_model, policy, cache: Optional[CacheConfig] = None):
        self.world, self.policy = world_model, policy
        self.cache = StateCache(cache)
        self.constraints = Constraints()
        self.internal_step = 0
        self.state_schema: Optional[Dict] = None
        self.action_schema: Optional[Dict] = None

    def set_environment(self, thermal: str, power: str) -> None:
        self.constraints = Constraints.from_thermal_power(thermal, power)

    def step(self, observations: List[Observation], horizon: int = 1) -> List[Any]:
        t0 = time.perf_counter()
        for o in observations:
            validate_observation(o, self.state_schema)
        now = _now_ms()
        self.cache.expire(now)
        self.cache.compress_old(now)
        h = self.constraints.effective_horizon(horizon)
        cur = self.cache.latest()
        skip = self.constraints.should_skip(self.internal_step)
        self.internal_step += 1
        if skip and cur is not None:  # degraded: reuse the current state, no new observation
            new, futures = cur, self.world.predict(cur, h)
            from_id = cur.state_id
        else:
            new, futures = self.world.observe(cur, observations, h)
            from_id = cur.state_id if cur else "init"
            self.cache.insert(new, "Normal")
        action = self.policy.decide(new, futures)
        validate_action(action, self.action_schema)
        chunks: List[Any] = [{"StateDelta": {"from_state_id": from_id, "to_state_id": new.state_id,
                                             "latent_update": None}}]
        chunks += [{"PredictedState": {"state_id": f.state_id, "confidence": f.confidence,
                                       "horizon_step": f.horizon_step}} for f in futures]
        chunks.append({"Action": {"action_space": action.action_space, "values": action.values}})
        chunks.append({"Metrics": {"compute_ms": int((time.perf_counter() - t0) * 1000)}})
        chunks.append("End")
        return chunks
