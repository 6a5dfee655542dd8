"""OpenAI- and Ollama-compatible HTTP server (FastAPI / uvicorn).

Routes (reference route table crates/server/src/lib.rs:2139-2244, 1811-1888):
  GET  /health  /ready (bloom.readiness v3)  /metrics (Prometheus)
  GET  /v1/models  /v1/models/{model}  /v1/observability  /v1/kv-cache-stats  /v1/backends
  POST /v1/chat/completions  /v1/completions  /v1/responses  /v1/embeddings  /v1/rerank
  GET  /v1/responses/{id}  /v1/responses/{id}/input_items
  POST /v1/cancel/{request_id}
  Ollama: GET /api/version /api/tags /api/ps, POST /api/show /api/chat /api/generate /api/embed /api/embeddings

Behaviour kept from the reference (README.md:494-664, lib.rs:141-189):
  * request limits (messages, stop sequences, max_tokens, embedding inputs, rerank documents, body size);
  * a full request semaphore answers 429 with `Retry-After: 1`;
  * every /v1 and /api response carries `x-request-id` (echoed when the client sent a valid one)
    and `Cache-Control: no-store`;
  * OpenAI-shaped errors on /v1, Ollama-shaped errors on /api, protocol-shaped 404/405;
  * chat streams start with an assistant-role chunk; `stream_options.include_usage` adds a final
    usage chunk before `data: [DONE]`; Ollama streams NDJSON;
  * stop sequences are filtered across deltas (never leak a partial match);
  * optional bearer API keys (`--api-key`), loopback-only unless keys are configured.
"""
from __future__ import annotations

import asyncio
import base64
import contextvars
import json
import os
import re
import struct
import time
import uuid
from collections import OrderedDict
from typing import Any, Dict, List, Optional

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse

from ..engine.chat_template import render
from ..engine.text import Detokenizer, StopSequenceFilter
from .metrics import Metrics
from .runtime import ServingRuntime

MAX_CHAT_MESSAGES = 2048
MAX_CHAT_CONTENT_BYTES = 768 * 1024
MAX_GENERATED_TOKENS = 32768
MAX_STOP_SEQUENCES = 4
MAX_STOP_SEQUENCE_CHARS = 1024
MAX_EMBEDDING_INPUTS = 256
MAX_RERANK_DOCUMENTS = 256
MAX_BODY_BYTES = 16 * 1024 * 1024
MAX_REQUEST_ID_CHARS = 128
READINESS_VERSION = 3
SERVER_VERSION = "0.1.0"
_RID = re.compile(r"^[A-Za-z0-9._:\-]{1,128}$")


class APIError(Exception):
    def __init__(self, status: int, message: str, type_: str = "invalid_request_error", param: Optional[str] = None,
                 code: Optional[str] = None, headers: Optional[dict] = None):
        super().__init__(message)
        self.status, self.message, self.type, self.param, self.code = status, message, type_, param, code
        self.headers = headers or {}


_EXPOSED = "x-request-id, retry-after, www-authenticate"
_LOOPBACK_HOSTS = ("127.0.0.1", "localhost", "[::1]", "::1")


def _split_origin(value: str):
    """(scheme, host, port) of a serialized browser origin, or None."""
    m = re.match(r"^(https?)://([^/:?#\s]+|\[[0-9a-fA-F:]+\])(?::(\d{1,5}))?$", value.strip())
    if not m:
        return None
    scheme, host, port = m.group(1), m.group(2).lower(), m.group(3)
    return scheme, host, int(port) if port else (443 if scheme == "https" else 80)


def origin_permitted(origins: List[str], loopback_listener: bool, origin_values: List[str], host_header: str) -> bool:
    """Browser-origin policy of the HTTP server.  No Origin header: a
    non-browser client, allowed.  Several Origin headers or an unparsable one
    ("null" included): refused.  `origins` ["*"] allows any origin, a list
    allows exactly those; otherwise only same-origin pages: an http origin
    whose host:port equals the request's Host, and a loopback host when the
    server listens on loopback only (DNS rebinding).  Reference:
    crates/server/src/lib.rs:283-320 (BrowserOriginGuard::permits)."""
    if not origin_values:
        return True
    if len(origin_values) > 1:
        return False
    o = _split_origin(origin_values[0])
    if o is None:
        return False
    if "*" in origins:
        return True
    if origin_values[0].strip().rstrip("/") in [x.rstrip("/") for x in origins]:
        return True
    scheme, host, port = o
    if scheme != "http":
        return False
    if loopback_listener and host not in _LOOPBACK_HOSTS:
        return False
    h = _split_origin("http://" + host_header.strip()) if host_header else None
    return h is not None and (h[1], h[2]) == (host, port)


def _cors_headers(resp, origins: List[str], origin: str) -> None:
    """Allowed cross-origin answer: "*" policy -> any origin; an exact list ->
    the configured origin the request matched (or the first one for a
    same-origin request); same-origin only -> no CORS header."""
    if "*" in origins:
        resp.headers["access-control-allow-origin"] = "*"
    elif origins:
        o = origin.strip().rstrip("/")
        resp.headers["access-control-allow-origin"] = o if o in [x.rstrip("/") for x in origins] else origins[0]
        resp.headers["vary"] = "Origin"
    else:
        return
    resp.headers["access-control-expose-headers"] = _EXPOSED


def _openai_error(e: APIError) -> JSONResponse:
    return JSONResponse({"error": {"message": e.message, "type": e.type, "param": e.param, "code": e.code}},
                        status_code=e.status, headers=e.headers)


def _ollama_error(e: APIError) -> JSONResponse:
    return JSONResponse({"error": e.message}, status_code=e.status, headers=e.headers)


class ResponseStore:
    """Process-local store of /v1/responses results: 256 records FIFO, 24 h
    (reference crates/server/src/response_store.rs:15-70)."""

    def __init__(self, cap: int = 256, ttl_s: float = 24 * 3600):
        self.cap, self.ttl = cap, ttl_s
        self.items: "OrderedDict[str, tuple]" = OrderedDict()

    def put(self, rid: str, resp: dict, inputs: list) -> None:
        self.items[rid] = (time.time(), resp, inputs)
        while len(self.items) > self.cap:
            self.items.popitem(last=False)

    def get(self, rid: str):
        v = self.items.get(rid)
        if v is None or time.time() - v[0] > self.ttl:
            return None
        return v


# The runtime-pool entry a request selected with its `model` field (set by
# check_model inside the request's own task; None = the default model).
_SELECTED: "contextvars.ContextVar" = contextvars.ContextVar("bloom_selected_runtime", default=None)


def _device_count() -> int:
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # pragma: no cover
        return 0


class _Ref:
    """Attribute proxy to the served pipeline / runtime: the entry this
    request selected from the runtime pool, else the swappable default."""

    def __init__(self, obj, attr: str):
        object.__setattr__(self, "_obj", obj)
        object.__setattr__(self, "_attr", attr)

    def _target(self):
        e = _SELECTED.get()
        if e is not None:
            return getattr(e, object.__getattribute__(self, "_attr"))
        return object.__getattribute__(self, "_obj")

    def __getattr__(self, k):
        return getattr(self._target(), k)

    def __setattr__(self, k, v):
        setattr(self._target(), k, v)

    def swap(self, obj) -> None:
        object.__setattr__(self, "_obj", obj)

    def get(self):
        return self._target()


class ServerSettings:
    def __init__(self, model_id: str = "model", api_keys: Optional[List[str]] = None, context_size: int = 2048,
                 max_concurrent: int = 4, allow_non_loopback: bool = False, cors_origins: Optional[List[str]] = None,
                 models_dir: Optional[str] = None, pool_capacity: int = 1, memory_host_limit: int = 0,
                 memory_device_limit: int = 0):
        self.model_id = model_id
        self.pool_capacity = int(pool_capacity)
        # aggregate byte budgets over every resident model (0 = physical RAM / device memory)
        self.memory_host_limit = int(memory_host_limit)
        self.memory_device_limit = int(memory_device_limit)
        self.api_keys = list(api_keys or [])
        self.context_size = context_size
        self.max_concurrent = max_concurrent
        self.allow_non_loopback = allow_non_loopback
        self.cors_origins = cors_origins or []
        self.models_dir = models_dir if models_dir is not None else os.environ.get("BLOOM_MODELS_DIR")
        # per-model token buckets (prompt + max_tokens per request), off unless BLOOM_RATE_LIMIT=1
        self.rate_limit = os.environ.get("BLOOM_RATE_LIMIT", "0") == "1"
        self.rate_limit_burst = float(os.environ.get("BLOOM_RATE_LIMIT_BURST", "32768"))
        self.rate_limit_rate = float(os.environ.get("BLOOM_RATE_LIMIT_RATE", "200"))

    @property
    def model_id(self) -> str:
        e = _SELECTED.get()
        return e.key if e is not None else self._model_id

    @model_id.setter
    def model_id(self, v: str) -> None:
        self._model_id = v

    @property
    def context_size(self) -> int:
        e = _SELECTED.get()
        if e is not None:
            return int(getattr(e.pipeline, "context_size", self._context_size))
        return self._context_size

    @context_size.setter
    def context_size(self, v: int) -> None:
        self._context_size = int(v)


def create_app(pipeline, settings: Optional[ServerSettings] = None, runtime: Optional[ServingRuntime] = None) -> FastAPI:
    st = settings or ServerSettings()
    metrics = Metrics()
    rt = runtime or ServingRuntime(pipeline, st.model_id, st.max_concurrent, metrics)
    rt.metrics = metrics
    from .._ext import runtime as _native

    limiter = _native().RateLimiter(st.rate_limit, st.rate_limit_burst, st.rate_limit_rate)
    # model management swaps the served pipeline / runtime behind these handles;
    # other resident models are selected per request through the runtime pool
    from .runtime_pool import (Footprint, KeepAliveError, MemoryBudget, MemoryError_, RuntimeEntry, RuntimePool,
                               parse_keep_alive)
    from ..utils.telemetry import MemoryTelemetry

    _mem = MemoryTelemetry.snapshot()
    budget = MemoryBudget(st.memory_host_limit or max(1, _mem.total_ram_bytes),
                          st.memory_device_limit or max(1, sum(d.total_bytes for d in _mem.devices) or 1 << 60))
    pool = RuntimePool(max(1, st.pool_capacity))
    # per-device accounting (C++ ResourceLedger): device -1 is host memory
    ledger = _native().ResourceLedger()
    ledger.add_device(-1, max(1, _mem.total_ram_bytes))
    for _d in _mem.devices:
        ledger.add_device(_d.index, _d.total_bytes)
    ledger_stamp = [0]
    pool.publish(RuntimeEntry(st.model_id, "", pipeline, rt), make_default=True)
    pipeline = _Ref(pipeline, "pipeline")
    rt = _Ref(rt, "runtime")
    store = ResponseStore()
    app = FastAPI(title="bloom_b200", version=SERVER_VERSION, docs_url=None, redoc_url=None, openapi_url=None)
    app.state.runtime = rt
    app.state.rate_limiter = limiter
    app.state.metrics = metrics
    started = time.time()
    def is_embedding() -> bool:
        return bool(getattr(pipeline, "is_embedding", False))

    # ------------------------------------------------------------ middleware
    @app.middleware("http")
    async def envelope(request: Request, call_next):
        path = request.url.path
        api = path.startswith("/v1") or path.startswith("/api")
        rid = request.headers.get("x-request-id")
        if not rid or not _RID.match(rid):
            rid = uuid.uuid4().hex
        request.state.request_id = rid
        origins = request.headers.getlist("origin")
        if not origin_permitted(st.cors_origins, not st.allow_non_loopback, origins, request.headers.get("host", "")):
            e = APIError(403, "The browser origin is not allowed by the Bloom server policy.", "invalid_request_error")
            resp = _ollama_error(e) if path.startswith("/api") else _openai_error(e)
            resp.headers["x-request-id"] = rid
            resp.headers["cache-control"] = "no-store"
            return resp
        if request.method == "OPTIONS" and origins and request.headers.get("access-control-request-method"):
            resp = Response(status_code=204)
            _cors_headers(resp, st.cors_origins, origins[0])
            resp.headers["access-control-allow-methods"] = "*"
            resp.headers["access-control-allow-headers"] = request.headers.get("access-control-request-headers", "*")
            resp.headers["x-request-id"] = rid
            return resp
        if api and st.api_keys:
            auth = request.headers.get("authorization", "")
            tok = auth[7:] if auth.lower().startswith("bearer ") else None
            if tok not in st.api_keys:
                e = APIError(401, "invalid or missing API key", "authentication_error",
                             headers={"WWW-Authenticate": 'Bearer realm="Bloom"'})
                resp = _ollama_error(e) if path.startswith("/api") else _openai_error(e)
                resp.headers["x-request-id"] = rid
                resp.headers["cache-control"] = "no-store"
                return resp
        cl = request.headers.get("content-length")
        if cl is not None and cl.isdigit() and int(cl) > MAX_BODY_BYTES:
            e = APIError(413, "request body too large")
            resp = _ollama_error(e) if path.startswith("/api") else _openai_error(e)
        else:
            metrics.requests_total += 1
            resp = await call_next(request)
        if api:
            resp.headers["x-request-id"] = rid
            resp.headers["cache-control"] = "no-store"
        if origins:
            _cors_headers(resp, st.cors_origins, origins[0])
        return resp

    @app.exception_handler(APIError)
    async def api_error(request: Request, e: APIError):
        metrics.errors_total += 1
        return _ollama_error(e) if request.url.path.startswith("/api") else _openai_error(e)

    from starlette.exceptions import HTTPException as StarletteHTTPException

    @app.exception_handler(StarletteHTTPException)
    async def http_error(request: Request, e: StarletteHTTPException):
        msg = "not found" if e.status_code == 404 else ("method not allowed" if e.status_code == 405 else str(e.detail))
        err = APIError(e.status_code, msg, "invalid_request_error" if e.status_code != 404 else "not_found_error")
        if request.url.path.startswith("/api"):
            return _ollama_error(err)
        return _openai_error(err)

    from fastapi.exceptions import RequestValidationError

    @app.exception_handler(RequestValidationError)
    async def validation_error(request: Request, e: RequestValidationError):
        err = APIError(400, f"invalid request: {e.errors()[:1]}")
        return _ollama_error(err) if request.url.path.startswith("/api") else _openai_error(err)

    async def body(request: Request) -> dict:
        try:
            d = await request.json()
        except Exception:
            raise APIError(400, "request body must be JSON")
        if not isinstance(d, dict):
            raise APIError(400, "request body must be a JSON object")
        return d

    # ------------------------------------------------------------ helpers
    def check_model(name: Optional[str]) -> None:
        """Select the resident model a request names (404 when none is)."""
        if name in (None, "") or name == st._model_id or st._model_id.endswith(str(name)):
            return
        e = pool.select(str(name))
        if e is None or e.key == pool.default_key:
            raise APIError(404, f"model {name!r} is not loaded", "not_found_error", "model", "model_not_found")
        _SELECTED.set(e)
        pool.touch(e.key)

    def sampling(d: dict, default_max: int = 128):
        from ..engine.engine import SamplingParams

        mt = d.get("max_completion_tokens", d.get("max_tokens", d.get("max_output_tokens", default_max)))
        if mt is None:
            mt = default_max
        if not isinstance(mt, int) or mt < 1 or mt > MAX_GENERATED_TOKENS:
            raise APIError(400, f"max_tokens must be an integer in [1, {MAX_GENERATED_TOKENS}]", param="max_tokens")
        temp = d.get("temperature", 0.7)
        top_p = d.get("top_p", 0.9)
        if not isinstance(temp, (int, float)) or not 0 <= temp <= 2:
            raise APIError(400, "temperature must be in [0, 2]", param="temperature")
        if not isinstance(top_p, (int, float)) or not 0 < top_p <= 1:
            raise APIError(400, "top_p must be in (0, 1]", param="top_p")
        seed = d.get("seed")
        mn = d.get("min_tokens", 0) or 0  # extension: no end-of-sequence before this many tokens
        if not isinstance(mn, int) or mn < 0:
            raise APIError(400, "min_tokens must be a non-negative integer", param="min_tokens")
        sp = SamplingParams(max_tokens=mt, temperature=float(temp), top_p=float(top_p), seed=seed,
                            top_k=int(d.get("top_k", 0) or 0), min_tokens=min(mn, mt))
        sp.segment = segment_of(d)
        return sp

    def segment_of(d: dict) -> int:
        """Request class for admission: OpenAI service_tier "flex" / "batch" ->
        background; "realtime" or Bloom's "segment" field by name; otherwise
        foreground interactive."""
        from .runtime import SEGMENTS

        seg = d.get("segment")
        if isinstance(seg, str):
            if seg not in SEGMENTS:
                raise APIError(400, f"segment must be one of {', '.join(SEGMENTS)}", param="segment")
            return SEGMENTS[seg]
        tier = d.get("service_tier")
        if tier in ("flex", "batch"):
            return SEGMENTS["background"]
        if tier == "realtime":
            return SEGMENTS["realtime"]
        return SEGMENTS["foreground"]

    def stops(d: dict) -> List[str]:
        s = d.get("stop")
        if s is None:
            return []
        if isinstance(s, str):
            s = [s]
        if not isinstance(s, list) or len(s) > MAX_STOP_SEQUENCES or any(
                not isinstance(x, str) or len(x) > MAX_STOP_SEQUENCE_CHARS for x in s):
            raise APIError(400, f"stop must be a string or up to {MAX_STOP_SEQUENCES} strings", param="stop")
        return s

    def messages_of(d: dict) -> List[Dict[str, str]]:
        msgs = d.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise APIError(400, "messages must be a non-empty array", param="messages")
        if len(msgs) > MAX_CHAT_MESSAGES:
            raise APIError(400, f"at most {MAX_CHAT_MESSAGES} messages", param="messages")
        if any(isinstance(m, dict) and (m.get("tool_calls") or m.get("role") == "tool") for m in msgs):
            from .tool_calling import ToolError, normalize_tool_history

            try:
                msgs = normalize_tool_history(msgs)
            except ToolError as e:
                raise APIError(400, str(e), param="messages") from None
        out, total = [], 0
        for m in msgs:
            if not isinstance(m, dict) or m.get("role") not in ("system", "user", "assistant", "tool", "developer"):
                raise APIError(400, "each message needs a role of system, user, assistant or tool", param="messages")
            c = m.get("content", "")
            if isinstance(c, list):
                c = "".join(p.get("text", "") for p in c if isinstance(p, dict) and p.get("type") in ("text", "input_text"))
            if c is None:
                c = ""
            if not isinstance(c, str):
                raise APIError(400, "message content must be a string or text parts", param="messages")
            total += len(c.encode("utf-8"))
            role = "system" if m["role"] == "developer" else m["role"]
            out.append({"role": role, "content": c})
        if total > MAX_CHAT_CONTENT_BYTES:
            raise APIError(413, "message content too large", param="messages")
        return out

    def prompt_ids_for(msgs: List[Dict[str, str]], raw_prompt: Optional[str] = None) -> List[int]:
        if raw_prompt is not None:
            ids = pipeline.tokenizer.encode(raw_prompt)
        else:
            ids = pipeline.tokenizer.encode(render(msgs, pipeline.template))
        if not ids:
            ids = [1]
        if len(ids) >= st.context_size:
            raise APIError(400, f"prompt has {len(ids)} tokens; the context window is {st.context_size}",
                           param="messages", code="context_length_exceeded")
        return ids

    def with_eos(params):
        eos = pipeline.eos_ids() if hasattr(pipeline, "eos_ids") else []
        params.stop_token_ids = list(set(params.stop_token_ids) | set(eos))
        return params

    async def token_stream(msgs, params, stop_list, request: Request, raw_prompt: Optional[str] = None,
                           prompt_ids: Optional[List[int]] = None, counter: Optional[dict] = None):
        """Yields (delta_text, finished, reason); handles admission, cancellation, stop strings.
        `counter["tokens"]` (if given) counts generated tokens."""
        if not state["loaded"]:
            raise APIError(503, "no model is loaded (model management unloaded it)", "server_error")
        want = (len(prompt_ids) if prompt_ids is not None else 0) + int(getattr(params, "max_tokens", 0) or 0)
        ok, wait = limiter.try_acquire(st.model_id, float(max(1, want)), time.monotonic())
        if not ok:
            import math

            raise APIError(429, f"token rate limit exceeded for {st.model_id}; retry in {wait:.1f} s",
                           "rate_limit_error", headers={"Retry-After": str(max(1, math.ceil(wait)))})
        if not rt.try_acquire():
            raise APIError(429, "server is at capacity; retry shortly", "rate_limit_error",
                           headers={"Retry-After": "1"})
        metrics.in_flight += 1
        sub = None
        try:
            if prompt_ids is not None:
                ids = list(prompt_ids)
                if len(ids) >= st.context_size:
                    raise APIError(400, f"prompt has {len(ids)} tokens; the context window is {st.context_size}",
                                   param="prompt", code="context_length_exceeded")
            else:
                ids = prompt_ids_for(msgs, raw_prompt)
            params.max_tokens = min(params.max_tokens, st.context_size - len(ids) - 1)
            with_eos(params)
            sub = rt.submit(ids, params, messages=None if rt.engine is not None else (raw_prompt or msgs),
                            request_id=request.state.request_id, segment=getattr(params, "segment", 0))
            detok = Detokenizer(pipeline.tokenizer)
            filt = StopSequenceFilter(stop_list)
            eos = set(pipeline.eos_ids()) if hasattr(pipeline, "eos_ids") else set()
            yield {"prompt_tokens": len(ids)}
            while True:
                item = await sub.queue.get()
                if item.error:
                    raise APIError(500, item.error, "server_error")
                if counter is not None and (item.token is not None or item.text):
                    counter["tokens"] = counter.get("tokens", 0) + 1
                delta = ""
                if item.token is not None and item.token not in eos:
                    delta = detok.add(item.token)
                elif item.text is not None:
                    delta = item.text
                out, stopped = filt.push(delta) if delta else ("", False)
                if stopped:
                    if not item.finished:
                        rt.cancel(sub.id)
                    yield (out, True, "stop")
                    return
                if item.finished:
                    out += filt.flush()
                    reason = item.reason if item.reason in ("stop", "length") else "stop"
                    yield (out, True, reason)
                    return
                if out:
                    yield (out, False, None)
                if await request.is_disconnected():
                    rt.cancel(sub.id)
                    return
        finally:
            metrics.in_flight -= 1
            rt.release()

    # ------------------------------------------------------------ health / readiness / metrics
    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/ready")
    async def ready():
        ok = rt.ready and rt.available_permits > 0
        snap = {"schema_version": READINESS_VERSION, "object": "bloom.readiness", "protocol_version": READINESS_VERSION,
                "minimum_ui_protocol_version": READINESS_VERSION, "maximum_ui_protocol_version": READINESS_VERSION,
                "server_version": SERVER_VERSION, "status": "ready" if ok else "busy", "progress": 100,
                "model": st.model_id, "loading": False, "load_error": None,
                "input_modalities": ["Text"], "model_tasks": ["embedding"] if is_embedding() else ["chat", "completion"],
                "context_window": st.context_size, "in_flight_requests": rt.in_flight,
                "available_permits": rt.available_permits, "memory_pressure_high": False,
                "ram_utilization": _ram_utilization()}
        return JSONResponse(snap, status_code=200 if ok else 503)

    def _sched_gauges() -> dict:
        eng = getattr(pipeline, "llm", None)
        sch = getattr(eng, "scheduler", None)
        if sch is None:
            return {}
        return {"waiting_requests": sch.num_waiting, "running_requests": sch.num_running,
                "preemptions_total": sch.total_preemptions, "admissions_deferred_total": sch.admissions_deferred,
                "failed_steps_total": len(getattr(eng, "failures", []))}

    def _memory():
        from ..utils.telemetry import MemoryTelemetry

        dev = getattr(getattr(pipeline, "llm", None), "model", None)
        idx = [dev.device.index] if dev is not None and getattr(dev.device, "index", None) is not None else []
        return MemoryTelemetry.snapshot(idx)

    @app.get("/metrics")
    async def prom():
        kv = _kv_stats(pipeline)
        return PlainTextResponse(metrics.render(kv, _sched_gauges(), _memory()),
                                 media_type="text/plain; version=0.0.4")

    @app.get("/v1/observability")
    async def observability():
        from ..utils import tracing

        return {"object": "bloom.observability", "schema_version": 1, "uptime_seconds": time.time() - started,
                "model": st.model_id, "metrics": metrics.snapshot(), "kv_cache": _kv_stats(pipeline),
                "scheduler": _sched_gauges(), "memory": _memory().to_dict(), "spans": tracing.stats(),
                "runtime": {"in_flight_requests": rt.in_flight, "available_permits": rt.available_permits,
                            "engine": getattr(pipeline, "engine_name", "unknown"), "broken": rt.broken}}

    @app.get("/v1/kv-cache-stats")
    async def kv_stats():
        return {"object": "kv_cache_stats", "pool": _kv_stats(pipeline), "cachemesh": _cachemesh_stats(pipeline)}

    @app.get("/v1/backends")
    async def backends():
        from ..engine.registry import default_registry

        return {"object": "list", "data": default_registry().describe()}

    # ------------------------------------------------------------ multimodal
    def _multipart(raw: bytes, ctype: str) -> Dict[str, tuple]:
        """name -> (bytes, content type) of a multipart/form-data body."""
        from email.parser import BytesParser
        from email.policy import HTTP

        msg = BytesParser(policy=HTTP).parsebytes(b"Content-Type: " + ctype.encode() + b"\r\n\r\n" + raw)
        if not msg.is_multipart():
            raise APIError(400, "expected a multipart/form-data upload")
        out = {}
        for part in msg.iter_parts():
            name = part.get_param("name", header="content-disposition")
            if name:
                out[str(name)] = (part.get_payload(decode=True) or b"", part.get_content_type())
        return out

    async def _multimodal(request: Request, blocks, params):
        from ..engine.processor import ProcessorError
        from ..engine.vl_pipeline import parse_blocks

        if not getattr(pipeline, "accepts_images", False):
            raise APIError(400, "the loaded model does not accept multimodal input", param="model")
        try:
            parse_blocks(blocks)  # fail before streaming starts
        except ProcessorError as e:
            raise APIError(400, str(e), param="blocks") from None
        if not rt.try_acquire():
            raise APIError(429, "server is at capacity; retry shortly", "rate_limit_error", headers={"Retry-After": "1"})
        loop = asyncio.get_running_loop()
        q: "asyncio.Queue" = asyncio.Queue()
        pipe = pipeline.get()

        def work():
            try:
                for d in pipe.run_multimodal(blocks, params):
                    loop.call_soon_threadsafe(q.put_nowait, ("delta", d))
                loop.call_soon_threadsafe(q.put_nowait, ("end", None))
            except Exception as e:  # noqa: BLE001 - reported in the stream
                loop.call_soon_threadsafe(q.put_nowait, ("error", str(e)))

        t0 = time.time()
        loop.run_in_executor(None, work)

        async def sse():
            n = 0
            try:
                while True:
                    kind, v = await q.get()
                    if kind == "delta":
                        n += 1
                        yield f"data: {json.dumps({'TextDelta': v})}\n\n"
                    elif kind == "error":
                        yield f"data: {json.dumps({'error': {'message': v, 'type': 'server_error'}})}\n\n"
                        return
                    else:
                        metrics.tokens_generated += n
                        yield f"data: {json.dumps({'Metrics': {'compute_ms': int((time.time() - t0) * 1000)}})}\n\n"
                        yield f"data: {json.dumps('End')}\n\n"
                        return
            finally:
                rt.release()

        return StreamingResponse(sse(), media_type="text/event-stream")

    @app.post("/v1/multimodal/stream")
    async def multimodal_stream(request: Request):
        """InferenceRequest {"blocks": [...], "params": {max_tokens, temperature,
        top_p, seed}} -> SSE of OutputChunks (TextDelta ..., Metrics, End)."""
        d = await body(request)
        check_model(d.get("model"))
        return await _multimodal(request, d.get("blocks"), sampling(d.get("params") or {}, 128))

    @app.post("/v1/multimodal/upload")
    async def multimodal_upload(request: Request):
        """multipart/form-data: prompt, image (image/png; JPEG is refused),
        optional model and max_tokens -> the same SSE stream."""
        raw = await request.body()
        if len(raw) > 32 * 1024 * 1024:
            raise APIError(413, "upload too large (32 MiB at most)")
        parts = _multipart(raw, request.headers.get("content-type", ""))
        if "model" in parts:
            check_model(parts["model"][0].decode("utf-8", "replace"))
        blocks = []
        if "image" in parts:
            data, mime = parts["image"]
            blocks.append({"Image": {"bytes": base64.b64encode(data).decode(), "mime": mime}})
        if "prompt" in parts:
            blocks.append({"Text": parts["prompt"][0].decode("utf-8", "replace")})
        p = {"max_tokens": int(parts["max_tokens"][0]) if "max_tokens" in parts else 512}
        return await _multimodal(request, blocks, sampling(p, 512))

    # ------------------------------------------------------------ world-model loop
    world_sessions: "OrderedDict[str, Any]" = OrderedDict()

    @app.post("/v1/world/step")
    async def world_step(request: Request):
        """One observation -> state -> predicted futures -> action cycle.
        Without `session` every call starts a fresh loop (the reference's
        behaviour); with `session` the loop and its state cache persist
        between calls (at most 64 sessions, least recently used dropped).
        `engine`: "latent" (GPU latent dynamics, the default) or "mock"."""
        from ..engine import world as W

        d = await body(request)
        try:
            obs = [W.Observation.parse(o) for o in (d.get("observations") or [])]
            horizon = d.get("horizon", 1)
            if not isinstance(horizon, int) or not 0 <= horizon <= 64:
                raise W.WorldError("horizon must be an integer in [0, 64]")
            sid = d.get("session")
            loop = world_sessions.get(sid) if sid else None
            if loop is None:
                cc = W.CacheConfig()
                for k, v in (d.get("cache_config") or {}).items():
                    if hasattr(cc, k) and v is not None:
                        setattr(cc, k, type(getattr(cc, k))(v))
                kind = d.get("engine", "latent")
                sp = (d.get("action_schema") or {}).get("allowed_action_spaces") or ["robot_velocity"]
                dim = (d.get("action_schema") or {}).get("action_dimensions", {}).get(sp[0], 2)
                if kind == "mock":
                    loop = W.WorldModelLoop(W.MockWorldModel(), W.MockPolicy(sp[0], dim), cc)
                elif kind == "latent":
                    loop = W.WorldModelLoop(W.LatentWorldModel(), W.LinearPolicy(action_space=sp[0], dim=dim), cc)
                else:
                    raise W.WorldError("engine must be latent or mock")
                if sid:
                    world_sessions[str(sid)] = loop
                    while len(world_sessions) > 64:
                        world_sessions.popitem(last=False)
            elif sid:
                world_sessions.move_to_end(str(sid))
            loop.state_schema = d.get("state_schema")
            loop.action_schema = d.get("action_schema")
            if d.get("thermal_state") is not None and d.get("power_state") is not None:
                loop.set_environment(str(d["thermal_state"]), str(d["power_state"]))
            chunks = await asyncio.get_running_loop().run_in_executor(None, loop.step, obs, horizon)
        except W.WorldError as e:
            raise APIError(400, str(e), "invalid_observation_or_action") from None
        if d.get("stream"):
            async def sse():
                for c in chunks:
                    yield f"data: {json.dumps(c)}\n\n"

            return StreamingResponse(sse(), media_type="text/event-stream")
        return chunks

    @app.post("/v1/cancel/{request_id}")
    async def cancel(request_id: str):
        if not rt.cancel(request_id):
            raise APIError(404, f"no in-flight request {request_id}", "not_found_error")
        return {"id": request_id, "object": "cancellation", "cancelled": True}

    # ------------------------------------------------------------ models
    def model_card():
        return {"id": st.model_id, "object": "model", "created": int(started), "owned_by": "bloom_b200"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [model_card()]}

    @app.get("/v1/models/{model:path}")
    async def model(model: str):
        check_model(model)
        return model_card()

    # ------------------------------------------------------------ function tools
    from .tool_calling import (ToolError, envelope_schema, finish_reason as tool_finish, parse_tool_output,
                               protocol_instruction, tool_calls_json, tool_config)

    def tool_setup(d: dict, msgs: List[Dict[str, str]], params, cfg=None):
        """Parse tools / tool_choice; with tools active, append the protocol
        instruction and constrain decoding to the JSON envelope."""
        try:
            if cfg is None:
                cfg = tool_config(d.get("tools"), d.get("tool_choice"), d.get("parallel_tool_calls"))
        except ToolError as e:
            raise APIError(400, str(e), param="tools") from None
        if cfg is None:
            return None
        msgs.append({"role": "system", "content": protocol_instruction(cfg)})
        params.json_mode = True
        params.json_schema = envelope_schema(cfg)
        return cfg

    def parse_tools_output(text: str, cfg):
        from ..engine.structured import repair_json

        try:
            return parse_tool_output(repair_json(text), cfg)
        except ToolError as e:
            raise APIError(502, f"model output did not follow the function-calling protocol: {e}",
                           "server_error") from None

    # ------------------------------------------------------------ chat / completions
    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        if is_embedding():
            raise APIError(400, "the loaded model is an embedding model", param="model")
        d = await body(request)
        check_model(d.get("model"))
        msgs = messages_of(d)
        params = sampling(d)
        stop_list = stops(d)
        rf = d.get("response_format")
        tools = tool_setup(d, msgs, params)
        if rf is not None and tools is None:
            from ..engine.structured import SchemaError, constrain_params

            try:
                constrain_params(params, rf, pipeline)
            except SchemaError as e:
                raise APIError(400, str(e), param="response_format") from None
        cid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        stream = bool(d.get("stream"))
        include_usage = bool((d.get("stream_options") or {}).get("include_usage"))
        gen = token_stream(msgs, params, stop_list, request)
        first = await gen.__anext__()  # admission / validation errors surface before streaming starts
        ptoks = first["prompt_tokens"]
        if not stream:
            text, reason, n = [], "stop", 0
            async for out, fin, r in gen:
                text.append(out)
                n += 1
                if fin:
                    reason = r
            content = "".join(text)
            metrics.tokens_generated += n
            if tools is not None:
                parsed = parse_tools_output(content, tools)
                msg = {"role": "assistant", "content": parsed.message}
                if parsed.is_calls:
                    msg["tool_calls"] = tool_calls_json(cid, parsed)
                return {"id": cid, "object": "chat.completion", "created": created, "model": st.model_id,
                        "choices": [{"index": 0, "message": msg, "logprobs": None,
                                     "finish_reason": tool_finish(parsed, n, params.max_tokens)}],
                        "usage": {"prompt_tokens": ptoks, "completion_tokens": n, "total_tokens": ptoks + n}}
            msg = {"role": "assistant", "content": content}
            if rf and rf.get("type") in ("json_object", "json_schema"):
                from ..engine.structured import repair_json

                msg["content"] = repair_json(content)
            return {"id": cid, "object": "chat.completion", "created": created, "model": st.model_id,
                    "choices": [{"index": 0, "message": msg, "logprobs": None, "finish_reason": reason}],
                    "usage": {"prompt_tokens": ptoks, "completion_tokens": n, "total_tokens": ptoks + n}}

        async def sse():
            def chunk(delta, reason=None):
                return {"id": cid, "object": "chat.completion.chunk", "created": created, "model": st.model_id,
                        "choices": [{"index": 0, "delta": delta, "logprobs": None, "finish_reason": reason}]}

            yield f"data: {json.dumps(chunk({'role': 'assistant', 'content': ''}))}\n\n"
            n = 0
            reason = "stop"
            buffered = []
            try:
                async for out, fin, r in gen:
                    n += 1
                    if out and tools is not None:
                        buffered.append(out)  # the envelope is parsed once complete
                    elif out:
                        yield f"data: {json.dumps(chunk({'content': out}))}\n\n"
                    if fin:
                        reason = r
                        break
                if tools is not None:
                    parsed = parse_tools_output("".join(buffered), tools)
                    delta = ({"tool_calls": tool_calls_json(cid, parsed, with_index=True)} if parsed.is_calls
                             else {"content": parsed.message})
                    metrics.tokens_generated += n
                    yield f"data: {json.dumps(chunk(delta, tool_finish(parsed, n, params.max_tokens)))}\n\n"
                    yield "data: [DONE]\n\n"
                    return
            except APIError as e:
                yield f"data: {json.dumps({'error': {'message': e.message, 'type': e.type}})}\n\n"
                yield "data: [DONE]\n\n"
                return
            metrics.tokens_generated += n
            yield f"data: {json.dumps(chunk({}, reason))}\n\n"
            if include_usage:
                u = {"id": cid, "object": "chat.completion.chunk", "created": created, "model": st.model_id,
                     "choices": [], "usage": {"prompt_tokens": ptoks, "completion_tokens": n,
                                              "total_tokens": ptoks + n}}
                yield f"data: {json.dumps(u)}\n\n"
            yield "data: [DONE]\n\n"

        return StreamingResponse(sse(), media_type="text/event-stream")

    @app.post("/v1/completions")
    async def completions(request: Request):
        if is_embedding():
            raise APIError(400, "the loaded model is an embedding model", param="model")
        d = await body(request)
        check_model(d.get("model"))
        prompt = d.get("prompt")
        token_prompt = None
        if isinstance(prompt, list) and prompt and all(isinstance(p, int) and not isinstance(p, bool) for p in prompt):
            token_prompt = prompt  # OpenAI form: the prompt as token ids
            vocab = getattr(getattr(pipeline, "cfg", None), "vocab_size", None)
            if vocab and any(p < 0 or p >= vocab for p in token_prompt):
                raise APIError(400, "prompt token id out of the vocabulary", param="prompt")
            prompt = ""
        elif isinstance(prompt, list):
            prompt = "".join(p for p in prompt if isinstance(p, str))
        if not isinstance(prompt, str):
            raise APIError(400, "prompt must be a string or a list of token ids", param="prompt")
        params = sampling(d, 16)
        stop_list = stops(d)
        cid = "cmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        counter = {"tokens": 0}
        gen = token_stream([{"role": "user", "content": prompt}], params, stop_list, request, raw_prompt=prompt,
                           prompt_ids=token_prompt, counter=counter)
        first = await gen.__anext__()
        ptoks = first["prompt_tokens"]
        if not d.get("stream"):
            text, reason, n = [], "stop", 0
            async for out, fin, r in gen:
                text.append(out)
                n += 1
                if fin:
                    reason = r
            n = counter["tokens"] or n
            metrics.tokens_generated += n
            return {"id": cid, "object": "text_completion", "created": created, "model": st.model_id,
                    "choices": [{"index": 0, "text": "".join(text), "logprobs": None, "finish_reason": reason}],
                    "usage": {"prompt_tokens": ptoks, "completion_tokens": n, "total_tokens": ptoks + n}}

        async def sse():
            n = 0
            async for out, fin, r in gen:
                n += 1
                c = {"id": cid, "object": "text_completion", "created": created, "model": st.model_id,
                     "choices": [{"index": 0, "text": out, "logprobs": None, "finish_reason": r if fin else None}]}
                yield f"data: {json.dumps(c)}\n\n"
                if fin:
                    break
            metrics.tokens_generated += n
            yield "data: [DONE]\n\n"

        return StreamingResponse(sse(), media_type="text/event-stream")

    # ------------------------------------------------------------ responses API
    @app.post("/v1/responses")
    async def responses(request: Request):
        d = await body(request)
        check_model(d.get("model"))
        inp = d.get("input")
        msgs = []
        if d.get("instructions"):
            msgs.append({"role": "system", "content": str(d["instructions"])})
        if isinstance(inp, str):
            msgs.append({"role": "user", "content": inp})
        elif isinstance(inp, list):
            msgs += messages_of({"messages": [m for m in inp if isinstance(m, dict) and "role" in m]})
        else:
            raise APIError(400, "input must be a string or a list of messages", param="input")
        params = sampling(d)
        rid = "resp_" + uuid.uuid4().hex[:24]
        mid = "msg_" + uuid.uuid4().hex[:24]
        created = int(time.time())
        from .tool_calling import responses_tool_config

        try:
            rcfg, echoed_tools, echoed_choice = responses_tool_config(d.get("tools"), d.get("tool_choice"),
                                                                      d.get("parallel_tool_calls"))
        except ToolError as e:
            raise APIError(400, str(e), param="tools") from None
        tools = tool_setup(d, msgs, params, cfg=rcfg) if rcfg is not None else None
        gen = token_stream(msgs, params, [], request)
        first = await gen.__anext__()
        ptoks = first["prompt_tokens"]

        def final(text, n, status="completed"):
            output = [{"type": "message", "id": mid, "status": "completed", "role": "assistant",
                       "content": [{"type": "output_text", "text": text, "annotations": []}]}]
            if tools is not None and status == "completed":
                parsed = parse_tools_output(text, tools)
                if parsed.is_calls:
                    output = [{"type": "function_call", "id": f"fc_{rid[5:]}_{i}", "call_id": cid_,
                               "name": c["function"]["name"], "arguments": c["function"]["arguments"],
                               "status": "completed"}
                              for i, (c, cid_) in enumerate((c, c["id"]) for c in tool_calls_json(rid, parsed))]
                else:
                    output[0]["content"][0]["text"] = parsed.message
            r = {"id": rid, "object": "response", "created_at": created, "status": status, "model": st.model_id,
                 "output": output, "usage": {"input_tokens": ptoks, "output_tokens": n, "total_tokens": ptoks + n}}
            if tools is not None or echoed_tools:
                r.update(tools=echoed_tools, tool_choice=echoed_choice,
                         parallel_tool_calls=bool(tools.parallel) if tools is not None else False)
            return r

        if not d.get("stream"):
            text, n = [], 0
            async for out, fin, r in gen:
                text.append(out)
                n += 1
            resp = final("".join(text), n)
            store.put(rid, resp, msgs)
            metrics.tokens_generated += n
            return resp

        async def sse():
            seq = 0

            def ev(kind, payload):
                nonlocal seq
                seq += 1
                payload = dict(payload, type=kind, sequence_number=seq)
                return f"event: {kind}\ndata: {json.dumps(payload)}\n\n"

            yield ev("response.created", {"response": dict(final("", 0, "in_progress"), output=[])})
            text, n = [], 0
            async for out, fin, r in gen:
                n += 1
                if out:
                    text.append(out)
                    if tools is None:  # a function-calling envelope is reported once parsed
                        yield ev("response.output_text.delta", {"item_id": mid, "output_index": 0,
                                                                "content_index": 0, "delta": out})
                if fin:
                    break
            full = "".join(text)
            resp = final(full, n)
            if tools is None:
                yield ev("response.output_text.done", {"item_id": mid, "output_index": 0, "content_index": 0,
                                                       "text": full})
            else:
                for i, item in enumerate(resp["output"]):
                    yield ev("response.output_item.done", {"output_index": i, "item": item})
            store.put(rid, resp, msgs)
            metrics.tokens_generated += n
            yield ev("response.completed", {"response": resp})

        return StreamingResponse(sse(), media_type="text/event-stream")

    @app.get("/v1/responses/{rid}")
    async def get_response(rid: str):
        v = store.get(rid)
        if v is None:
            raise APIError(404, f"response {rid} not found", "not_found_error")
        return v[1]

    @app.get("/v1/responses/{rid}/input_items")
    async def get_inputs(rid: str):
        v = store.get(rid)
        if v is None:
            raise APIError(404, f"response {rid} not found", "not_found_error")
        items = [{"type": "message", "role": m["role"], "content": [{"type": "input_text", "text": m["content"]}]}
                 for m in v[2]]
        return {"object": "list", "data": items}

    # ------------------------------------------------------------ embeddings / rerank
    def embed(texts: List[str], dims: Optional[int] = None) -> List[List[float]]:
        if not is_embedding():
            raise APIError(400, "the loaded model does not produce embeddings", param="model")
        return pipeline.embedder.embed(texts, dimensions=dims)

    @app.post("/v1/embeddings")
    async def embeddings(request: Request):
        d = await body(request)
        check_model(d.get("model"))
        inp = d.get("input")
        if isinstance(inp, str):
            inp = [inp]
        if not isinstance(inp, list) or not inp or len(inp) > MAX_EMBEDDING_INPUTS or \
                not all(isinstance(x, str) and x for x in inp):
            raise APIError(400, f"input must be a non-empty string or 1..{MAX_EMBEDDING_INPUTS} non-empty strings",
                           param="input")
        dims = d.get("dimensions")
        if dims is not None and (not isinstance(dims, int) or dims < 1):
            raise APIError(400, "dimensions must be a positive integer", param="dimensions")
        vecs = await asyncio.get_running_loop().run_in_executor(None, embed, inp, dims)
        fmt = d.get("encoding_format", "float")
        data = []
        for i, v in enumerate(vecs):
            e = base64.b64encode(struct.pack(f"<{len(v)}f", *v)).decode() if fmt == "base64" else v
            data.append({"object": "embedding", "index": i, "embedding": e})
        n = sum(len(x.split()) for x in inp)
        return {"object": "list", "data": data, "model": st.model_id, "usage": {"prompt_tokens": n, "total_tokens": n}}

    @app.post("/v1/rerank")
    async def rerank(request: Request):
        d = await body(request)
        q = d.get("query")
        docs = d.get("documents")
        if not isinstance(q, str) or not q:
            raise APIError(400, "query must be a non-empty string", param="query")
        if not isinstance(docs, list) or not docs or len(docs) > MAX_RERANK_DOCUMENTS:
            raise APIError(400, f"documents must hold 1..{MAX_RERANK_DOCUMENTS} items", param="documents")
        texts = [x if isinstance(x, str) else (x or {}).get("text", "") for x in docs]
        vecs = await asyncio.get_running_loop().run_in_executor(None, embed, [q] + texts, None)
        qv = vecs[0]
        scores = [sum(a * b for a, b in zip(qv, v)) for v in vecs[1:]]
        order = sorted(range(len(scores)), key=lambda i: (-scores[i], i))  # stable ties by index
        top = d.get("top_n") or len(order)
        res = [{"index": i, "relevance_score": scores[i], "document": {"text": texts[i]}} for i in order[:top]]
        return {"object": "list", "model": st.model_id, "results": res}

    # ------------------------------------------------------------ Ollama adapter
    # ------------------------------------------------------------ model management (operator API)
    from .catalog import ModelCatalog

    catalog = ModelCatalog(st.models_dir)
    state = {"loaded": True}

    def require_catalog():
        if catalog.root is None:
            raise APIError(404, "no models directory is configured (--models-dir / BLOOM_MODELS_DIR)",
                           "not_found_error")

    @app.get("/v1/model-management/models")
    async def mm_list():
        require_catalog()
        return {"object": "list", "data": catalog.entries(), "active": st.model_id if state["loaded"] else None}

    @app.post("/v1/model-management/preflight")
    async def mm_preflight(request: Request):
        require_catalog()
        d = await body(request)
        try:
            return catalog.preflight(str(d.get("model", "")), int(d.get("context_size", st.context_size)),
                                     int(d.get("max_concurrent", st.max_concurrent)), int(d.get("tp", 1)))
        except KeyError:
            raise APIError(404, f"model {d.get('model')!r} is not in the catalog", "not_found_error", "model",
                           "model_not_found")

    @app.post("/v1/model-management/switch")
    async def mm_switch(request: Request):
        require_catalog()
        d = await body(request)
        e = catalog.find(str(d.get("model", "")))
        if e is None or not e.get("valid"):
            raise APIError(404, f"model {d.get('model')!r} is not a loadable catalog entry", "not_found_error",
                           "model", "model_not_found")
        loader = getattr(app.state, "model_loader", None)
        if loader is None:
            raise APIError(501, "this server was started without a model loader", "server_error")
        if rt.in_flight:
            raise APIError(409, "requests are in flight; retry when idle", "conflict")
        import asyncio

        entry = await load_entry(e, make_default=True)
        st.model_id = entry.key
        st.context_size = int(getattr(entry.pipeline, "context_size", st.context_size))
        pipeline.swap(entry.pipeline)
        rt.swap(entry.runtime)
        state["loaded"] = True
        return {"status": "switched", "model": st.model_id}

    def footprint_of(e: dict) -> "Footprint":
        """Memory the model will hold: the manifest estimate for the server's context and concurrency."""
        try:
            pf = catalog.preflight(str(e["id"]), st._context_size, st.max_concurrent)
            total = int(pf.get("total_bytes", 0) or 0)
        except Exception:  # noqa: BLE001 - an unestimable package is charged its file size
            total = int(e.get("size_bytes", 0) or 0)
        on_gpu = _device_count() > 0
        return Footprint(host_bytes=0 if on_gpu else total, device_bytes=total if on_gpu else 0)

    async def load_entry(e: dict, make_default: bool = False, keep_alive_s: Optional[float] = None) -> "RuntimeEntry":
        """Load a catalog entry under a memory permit and publish it in the pool
        (idle least-recently-used residents are evicted to make room)."""
        loader = getattr(app.state, "model_loader", None)
        if loader is None:
            raise APIError(501, "this server was started without a model loader", "server_error")
        key = str(e["id"])
        fp = footprint_of(e)
        old = pool.get(key)
        if old is not None and old.permit is not None:
            old.permit.release()  # a reload replaces the old generation's charge
            old.permit = None
        for v in pool.evict_for(budget, fp, protect=key):
            metrics_evictions[0] += 1
        try:
            permit = budget.reserve(fp)
        except MemoryError_ as ex:
            raise APIError(507, f"model {key!r} does not fit the memory budget: {ex}", "server_error") from None
        dev = 0 if fp.device_bytes else -1
        ledger_stamp[0] += 1
        ok, evicted = ledger.reserve(key, dev, fp.device_bytes or fp.host_bytes, 2 if make_default else 1,
                                     ledger_stamp[0])
        if not ok:
            permit.release()
            raise APIError(507, f"model {key!r} does not fit device {dev}'s free memory", "server_error")
        for owner in evicted:  # lower-priority residents the ledger displaced
            v = pool.remove(owner)
            if v is not None:
                v.retire()
                metrics_evictions[0] += 1
        try:
            new_pipe = await asyncio.get_running_loop().run_in_executor(None, loader, e["path"])
        except Exception:
            permit.release()
            ledger.release(key)
            raise
        entry = RuntimeEntry(key, str(e["path"]), new_pipe, ServingRuntime(new_pipe, key, st.max_concurrent, metrics),
                             permit, on_retire=[ledger.release])
        if keep_alive_s is not None:
            entry.keep_alive_s = keep_alive_s
        for r in pool.publish(entry, make_default=make_default):
            if r is not entry:
                r.retire()
        pool.touch(key)
        return entry

    metrics_evictions = [0]

    @app.post("/v1/model-management/load")
    async def mm_load(request: Request):
        """Make another catalog model resident next to the default one; requests
        select it with their `model` field."""
        require_catalog()
        d = await body(request)
        e = catalog.find(str(d.get("model", "")))
        if e is None or not e.get("valid"):
            raise APIError(404, f"model {d.get('model')!r} is not a loadable catalog entry", "not_found_error",
                           "model", "model_not_found")
        try:
            ka = parse_keep_alive(d["keep_alive"]) if d.get("keep_alive") is not None else None
        except KeepAliveError as ex:
            raise APIError(400, str(ex), param="keep_alive") from None
        entry = await load_entry(e, keep_alive_s=ka)
        return {"status": "loaded", "model": entry.key, "resident": [x.key for x in pool.entries()]}

    @app.get("/v1/model-management/residency")
    async def mm_residency():
        return {"object": "bloom.residency", "capacity": pool.capacity, "default": pool.default_key,
                "memory_budget": budget.snapshot(), "evictions": metrics_evictions[0],
                "ledger": {str(dv): {"used_bytes": ledger.used(dv), "free_bytes": ledger.free_bytes(dv)}
                           for dv in [-1] + [d.index for d in _mem.devices]},
                "models": [{"model": x.key, "default": x.key == pool.default_key, "source": x.source,
                            "keep_alive_seconds": x.keep_alive_s,
                            "expires_at": _iso(x.expires_at) if x.expires_at else None,
                            "host_bytes": x.permit.footprint.host_bytes if x.permit else 0,
                            "device_bytes": x.permit.footprint.device_bytes if x.permit else 0,
                            "in_flight": getattr(x.runtime, "in_flight", 0)} for x in pool.entries()]}

    @app.post("/v1/model-management/unload")
    async def mm_unload(request: Request):
        d = await body(request) if (await request.body()) else {}
        key = d.get("model")
        if key and key != st._model_id:
            e = pool.get(str(key))
            if e is None:
                raise APIError(404, f"model {key!r} is not resident", "not_found_error", "model", "model_not_found")
            if getattr(e.runtime, "in_flight", 0):
                raise APIError(409, "requests are in flight; retry when idle", "conflict")
            pool.remove(e.key)
            e.retire()
            return {"status": "unloaded", "model": e.key}
        if rt.in_flight:
            raise APIError(409, "requests are in flight; retry when idle", "conflict")
        state["loaded"] = False
        return {"status": "unloaded", "model": st.model_id}

    async def expire_residents():
        """Keep-alive deadlines: unload residents whose deadline passed."""
        while True:
            await asyncio.sleep(0.25)
            for key in pool.expired():
                if key == pool.default_key:
                    e = pool.get(key)
                    if e is not None:
                        e.expires_at = None
                    state["loaded"] = False
                    continue
                e = pool.remove(key)
                if e is not None:
                    e.retire()

    @app.on_event("startup")
    async def _start_expiry():
        app.state.expiry_task = asyncio.get_running_loop().create_task(expire_residents())

    @app.on_event("shutdown")
    async def _stop_expiry():
        t = getattr(app.state, "expiry_task", None)
        if t is not None:
            t.cancel()

    @app.delete("/v1/model-management/models/{model_id}")
    async def mm_remove(model_id: str, confirm: bool = False):
        require_catalog()
        if not confirm:
            raise APIError(400, "removing model files needs ?confirm=true", param="confirm")
        if model_id == st.model_id and state["loaded"]:
            raise APIError(409, "the active model cannot be removed; switch or unload first", "conflict")
        try:
            catalog.remove(model_id)
        except KeyError:
            raise APIError(404, f"model {model_id!r} is not in the catalog", "not_found_error", "model",
                           "model_not_found")
        return {"status": "removed", "model": model_id}

    # ------------------------------------------------------------ acquisition (offline subset)
    def model_store():
        require_catalog()
        from .model_store import ModelStore

        if not hasattr(app.state, "model_store"):
            app.state.model_store = ModelStore(catalog.root)
        return app.state.model_store

    async def in_thread(fn, *a):
        from .model_store import StoreError

        try:
            return await asyncio.get_running_loop().run_in_executor(None, fn, *a)
        except StoreError as e:
            raise APIError(400, str(e)) from None

    @app.post("/v1/model-management/import")
    async def mm_import(request: Request):
        """Copy a local model file / package into the models directory with a
        checksum record (optionally checked against an expected sha256)."""
        d = await body(request)
        if not isinstance(d.get("path"), str):
            raise APIError(400, "import needs a local `path`", param="path")
        return await in_thread(model_store().import_package, d["path"], d.get("model"), d.get("sha256"))

    @app.post("/v1/model-management/record")
    async def mm_record(request: Request):
        d = await body(request)
        return await in_thread(model_store().record, str(d.get("model", "")), str(d.get("source", "local")))

    @app.post("/v1/model-management/verify")
    async def mm_verify(request: Request):
        d = await body(request)
        mid = str(d.get("model", ""))
        if mid == st._model_id and state["loaded"] and d.get("quarantine", True):
            raise APIError(409, "the active model cannot be quarantined; switch or unload first", "conflict")
        return await in_thread(model_store().verify, mid, bool(d.get("quarantine", True)))

    @app.get("/v1/model-management/integrity")
    async def mm_integrity():
        return model_store().status

    @app.get("/v1/model-management/inventory")
    async def mm_inventory():
        return model_store().inventory()

    @app.post("/v1/model-management/inventory/reconcile")
    async def mm_reconcile(request: Request):
        d = await body(request)
        return model_store().reconcile(d.get("inventory", d))

    @app.get("/v1/model-management/quarantine")
    async def mm_quarantine():
        return {"object": "list", "data": model_store().quarantined()}

    @app.post("/api/pull")
    async def ollama_pull(request: Request):
        return _ollama_error(APIError(501, "model downloads are not available in this offline build; copy the "
                                           "model package into the models directory instead"))

    @app.delete("/api/delete")
    async def ollama_delete(request: Request):
        try:
            require_catalog()
            d = await body(request)
            name = str(d.get("model") or d.get("name") or "")
            if name == st.model_id and state["loaded"]:
                raise APIError(409, "the active model cannot be removed")
            catalog.remove(name)
        except APIError as e:
            return _ollama_error(e)
        except KeyError:
            return _ollama_error(APIError(404, f"model '{name}' not found"))
        return JSONResponse({})

    @app.get("/api/version")
    async def o_version():
        return {"version": SERVER_VERSION}

    def o_model():
        return {"name": st.model_id, "model": st.model_id, "modified_at": _iso(started), "size": 0,
                "digest": uuid.uuid5(uuid.NAMESPACE_URL, st.model_id).hex,
                "details": {"format": "bloom", "family": getattr(pipeline.cfg, "arch", ""),
                            "parameter_size": "", "quantization_level": ""}}

    @app.get("/api/tags")
    async def o_tags():
        return {"models": [o_model()]}

    @app.get("/api/ps")
    async def o_ps():
        out = []
        for x in pool.entries():
            if x.key == pool.default_key and not state["loaded"]:
                continue
            exp = x.expires_at if x.expires_at is not None else (
                time.time() + 365 * 24 * 3600 if x.keep_alive_s < 0 else time.time() + x.keep_alive_s)
            out.append({"name": x.key, "model": x.key, "size": (x.permit.footprint.host_bytes +
                                                                x.permit.footprint.device_bytes) if x.permit else 0,
                        "digest": uuid.uuid5(uuid.NAMESPACE_URL, x.key).hex, "expires_at": _iso(exp),
                        "size_vram": x.permit.footprint.device_bytes if x.permit else 0,
                        "details": {"format": "bloom", "family": getattr(x.pipeline.cfg, "arch", "")}})
        return {"models": out}

    @app.post("/api/show")
    async def o_show(request: Request):
        d = await body(request)
        check_model(d.get("model") or d.get("name"))
        cfg = pipeline.cfg
        return {"modelfile": "", "parameters": "", "template": pipeline.template,
                "details": o_model()["details"],
                "model_info": {"general.architecture": cfg.arch, "context_length": st.context_size,
                               "embedding_length": cfg.hidden_size, "block_count": cfg.num_layers}}

    def o_params(d: dict):
        opts = d.get("options") or {}
        m = {"max_tokens": opts.get("num_predict", 128), "temperature": opts.get("temperature", 0.8),
             "top_p": opts.get("top_p", 0.9), "seed": opts.get("seed"), "top_k": opts.get("top_k", 0)}
        if m["max_tokens"] in (None, -1):
            m["max_tokens"] = 128
        return sampling(m), stops({"stop": opts.get("stop")})

    async def o_generate_common(request: Request, msgs, raw_prompt, chat_mode: bool, d: dict):
        params, stop_list = o_params(d)
        t0 = time.time()
        gen = token_stream(msgs, params, stop_list, request, raw_prompt=raw_prompt)
        first = await gen.__anext__()
        ptoks = first["prompt_tokens"]

        def piece(text, done, reason=None, n=0):
            base = {"model": st.model_id, "created_at": _iso(time.time()), "done": done}
            if chat_mode:
                base["message"] = {"role": "assistant", "content": text}
            else:
                base["response"] = text
            if done:
                dur = int((time.time() - t0) * 1e9)
                base.update(done_reason=reason or "stop", total_duration=dur, load_duration=0,
                            prompt_eval_count=ptoks, eval_count=n, eval_duration=dur)
            return base

        if d.get("stream", True):
            async def nd():
                n = 0
                async for out, fin, r in gen:
                    n += 1
                    if out:
                        yield json.dumps(piece(out, False)) + "\n"
                    if fin:
                        yield json.dumps(piece("", True, r, n)) + "\n"
                        break
                metrics.tokens_generated += n

            return StreamingResponse(nd(), media_type="application/x-ndjson")
        text, n, reason = [], 0, "stop"
        async for out, fin, r in gen:
            text.append(out)
            n += 1
            if fin:
                reason = r
        metrics.tokens_generated += n
        res = piece("".join(text), True, reason, n)
        return res

    async def o_resident(d: dict):
        """Ollama residency: the named model is made resident on demand (from
        the catalog), its keep_alive deadline is re-armed after the request,
        and an empty request with keep_alive only loads / unloads.  Returns
        (keep_alive seconds, lifecycle response or None)."""
        try:
            ka = parse_keep_alive(d.get("keep_alive"))
        except KeepAliveError as ex:
            raise APIError(400, str(ex), param="keep_alive") from None
        name = d.get("model") or d.get("name")
        if name and pool.select(str(name)) is None and not (name == st._model_id or st._model_id.endswith(str(name))):
            e = catalog.find(str(name)) if catalog.root else None
            if e is None or not e.get("valid"):
                raise APIError(404, f"model '{name}' not found", "not_found_error")
            await load_entry(e, keep_alive_s=ka)
        check_model(name)
        key = st.model_id
        empty = not d.get("messages") and not d.get("prompt")
        if empty:
            if ka == 0:
                e = pool.get(key)
                if e is not None and key != pool.default_key:
                    pool.remove(key)
                    e.retire()
                else:
                    state["loaded"] = False
                return ka, {"model": key, "created_at": _iso(time.time()), "done": True, "done_reason": "unload"}
            if key == pool.default_key:
                state["loaded"] = True
            pool.touch(key, ka)
            return ka, {"model": key, "created_at": _iso(time.time()), "done": True, "done_reason": "load"}
        return ka, None

    @app.post("/api/chat")
    async def o_chat(request: Request):
        d = await body(request)
        ka, life = await o_resident(d)
        if life is not None:
            if life["done_reason"] == "load":
                life["message"] = {"role": "assistant", "content": ""}
            return life
        msgs = messages_of({"messages": d.get("messages")})
        try:
            return await o_generate_common(request, msgs, None, True, d)
        finally:
            pool.touch(st.model_id, ka)

    @app.post("/api/generate")
    async def o_generate(request: Request):
        d = await body(request)
        ka, life = await o_resident(d)
        if life is not None:
            if life["done_reason"] == "load":
                life["response"] = ""
            return life
        try:
            return await o_generate_inner(request, d)
        finally:
            pool.touch(st.model_id, ka)

    async def o_generate_inner(request: Request, d: dict):
        p = d.get("prompt")
        if not isinstance(p, str):
            raise APIError(400, "prompt must be a string")
        if d.get("raw"):
            return await o_generate_common(request, [{"role": "user", "content": p}], p, False, d)
        msgs = ([{"role": "system", "content": d["system"]}] if d.get("system") else []) + \
            [{"role": "user", "content": p}]
        return await o_generate_common(request, msgs, None, False, d)

    @app.post("/api/embed")
    async def o_embed(request: Request):
        d = await body(request)
        check_model(d.get("model"))
        inp = d.get("input")
        if isinstance(inp, str):
            inp = [inp]
        if not isinstance(inp, list) or not inp or len(inp) > MAX_EMBEDDING_INPUTS:
            raise APIError(400, "input must be a string or a list of strings")
        vecs = await asyncio.get_running_loop().run_in_executor(None, embed, inp, d.get("dimensions"))
        return {"model": st.model_id, "embeddings": vecs}

    @app.post("/api/embeddings")
    async def o_embeddings(request: Request):
        d = await body(request)
        p = d.get("prompt")
        if not isinstance(p, str) or not p:
            raise APIError(400, "prompt must be a non-empty string")
        vecs = await asyncio.get_running_loop().run_in_executor(None, embed, [p], None)
        return {"embedding": vecs[0]}

    return app


def _iso(t: float) -> str:
    return time.strftime("%Y-%m-%dT%H:%M:%S", time.gmtime(t)) + f".{int((t % 1) * 1e6):06d}Z"


def _ram_utilization() -> float:
    try:
        tot = avail = None
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    tot = int(line.split()[1])
                elif line.startswith("MemAvailable:"):
                    avail = int(line.split()[1])
        if tot and avail is not None:
            return round(1.0 - avail / tot, 4)
    except OSError:
        pass
    return 0.0


def _kv_stats(pipeline) -> dict:
    llm = getattr(pipeline, "llm", None)
    if llm is None:
        return {"total_blocks": 0, "free_blocks": 0, "active_blocks": 0, "cached_blocks": 0, "hits": 0, "misses": 0,
                "evictions": 0, "reuses": 0}
    return llm.kv_metrics()


def _cachemesh_stats(pipeline) -> dict:
    mesh = getattr(getattr(pipeline, "llm", None), "cachemesh", None)
    return mesh.metrics() if mesh is not None else {"enabled": False}
