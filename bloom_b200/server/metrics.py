"""Prometheus metrics for the HTTP server.

Counters (requests, completed, failed, generated and prompt tokens), gauges
(in-flight requests, uptime, scheduler queues, KV pool, process / system /
GPU memory from utils.telemetry) and summaries over the 4,096 most recent
samples of time to first token, inter-token latency and whole-request
latency.  Reference: crates/server/src/metrics.rs:13-120 (counters, bounded
observation vectors, Prometheus text rendering).
"""
from __future__ import annotations

import collections
import threading
import time


class Metrics:
    def __init__(self, cap: int = 4096):
        self.started = time.time()
        self.requests_total = 0
        self.errors_total = 0
        self.requests_completed = 0
        self.requests_failed = 0
        self.tokens_generated = 0
        self.prompt_tokens = 0
        self.in_flight = 0
        self._ttft = collections.deque(maxlen=cap)
        self._itl = collections.deque(maxlen=cap)
        self._latency = collections.deque(maxlen=cap)
        self._lock = threading.Lock()

    def observe_ttft(self, s: float) -> None:
        with self._lock:
            self._ttft.append(s)

    def observe_itl(self, s: float) -> None:
        with self._lock:
            self._itl.append(s)

    def observe_request(self, latency_s: float, ok: bool, prompt_tokens: int = 0) -> None:
        with self._lock:
            self._latency.append(latency_s)
            if ok:
                self.requests_completed += 1
            else:
                self.requests_failed += 1
            self.prompt_tokens += int(prompt_tokens)

    @staticmethod
    def _quantiles(xs):
        if not xs:
            return {"p50": 0.0, "p90": 0.0, "p99": 0.0, "count": 0, "sum": 0.0}
        s = sorted(xs)

        def q(f):
            return s[min(len(s) - 1, int(f * (len(s) - 1)))]

        return {"p50": q(0.5), "p90": q(0.9), "p99": q(0.99), "count": len(s), "sum": float(sum(s))}

    def snapshot(self) -> dict:
        with self._lock:
            tt, it, lat = list(self._ttft), list(self._itl), list(self._latency)
        return {"requests_total": self.requests_total, "errors_total": self.errors_total,
                "requests_completed_total": self.requests_completed, "requests_failed_total": self.requests_failed,
                "tokens_generated_total": self.tokens_generated, "prompt_tokens_total": self.prompt_tokens,
                "in_flight_requests": self.in_flight, "uptime_seconds": round(time.time() - self.started, 3),
                "ttft_seconds": self._quantiles(tt), "inter_token_latency_seconds": self._quantiles(it),
                "request_latency_seconds": self._quantiles(lat)}

    def render(self, kv: dict, scheduler: dict = None, memory=None) -> str:
        s = self.snapshot()
        out = []

        def metric(name, kind, help_, value, labels=""):
            out.append(f"# HELP {name} {help_}")
            out.append(f"# TYPE {name} {kind}")
            out.append(f"{name}{labels} {value}")

        metric("bloom_requests_total", "counter", "HTTP requests received.", s["requests_total"])
        metric("bloom_errors_total", "counter", "Requests answered with an error.", s["errors_total"])
        metric("bloom_requests_completed_total", "counter", "Generation requests that finished.",
               s["requests_completed_total"])
        metric("bloom_requests_failed_total", "counter", "Generation requests that ended with an error.",
               s["requests_failed_total"])
        metric("bloom_tokens_generated_total", "counter", "Generated tokens.", s["tokens_generated_total"])
        metric("bloom_prompt_tokens_total", "counter", "Prompt tokens of finished requests.",
               s["prompt_tokens_total"])
        metric("bloom_in_flight_requests", "gauge", "Requests being served.", s["in_flight_requests"])
        metric("bloom_uptime_seconds", "gauge", "Seconds since the server started.", s["uptime_seconds"])
        for key, name, help_ in (("ttft_seconds", "bloom_ttft_seconds", "Time to first token."),
                                 ("inter_token_latency_seconds", "bloom_inter_token_latency_seconds",
                                  "Time between consecutive streamed tokens."),
                                 ("request_latency_seconds", "bloom_request_latency_seconds",
                                  "Submission to last token.")):
            v = s[key]
            out.append(f"# HELP {name} {help_} (recent samples)")
            out.append(f"# TYPE {name} summary")
            for q, lab in (("p50", "0.5"), ("p90", "0.9"), ("p99", "0.99")):
                out.append(f'{name}{{quantile="{lab}"}} {v[q]}')
            out.append(f"{name}_sum {v['sum']}")
            out.append(f"{name}_count {v['count']}")
        for k, v in (kv or {}).items():
            if isinstance(v, (int, float)):
                out.append(f"# TYPE bloom_kv_{k} gauge")
                out.append(f"bloom_kv_{k} {v}")
        if kv and kv.get("total_blocks"):
            metric("bloom_kv_cache_utilization", "gauge", "Fraction of KV blocks held by requests.",
                   round(kv.get("active_blocks", 0) / kv["total_blocks"], 6))
        for k, v in (scheduler or {}).items():
            metric(f"bloom_scheduler_{k}", "gauge", f"Scheduler {k.replace('_', ' ')}.", v)
        if memory is not None:
            metric("bloom_process_resident_memory_bytes", "gauge", "Resident set size.", memory.rss_bytes)
            metric("bloom_process_peak_resident_memory_bytes", "gauge", "Peak resident set size.",
                   memory.peak_rss_bytes)
            metric("bloom_system_memory_total_bytes", "gauge", "System RAM.", memory.total_ram_bytes)
            metric("bloom_system_memory_used_bytes", "gauge", "System RAM in use.",
                   memory.total_ram_bytes - memory.available_ram_bytes)
            metric("bloom_memory_pressure_high", "gauge", "RAM or a GPU above 85 % used.", int(memory.high_pressure))
            for dv in memory.devices:
                lab = f'{{device="{dv.index}"}}'
                out.append("# TYPE bloom_gpu_memory_used_bytes gauge")
                out.append(f"bloom_gpu_memory_used_bytes{lab} {dv.used_bytes}")
                out.append("# TYPE bloom_gpu_memory_total_bytes gauge")
                out.append(f"bloom_gpu_memory_total_bytes{lab} {dv.total_bytes}")
                out.append("# TYPE bloom_gpu_memory_peak_bytes gauge")
                out.append(f"bloom_gpu_memory_peak_bytes{lab} {dv.peak_bytes}")
        return "\n".join(out) + "\n"
