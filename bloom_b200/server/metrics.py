"""Prometheus metrics: request/token/in-flight counters and bounded latency samples
(4,096 most recent TTFT / inter-token / request latencies; reference
crates/server/src/metrics.rs:13-120), plus the KV-pool gauges."""
from __future__ import annotations

import collections
import statistics
import threading


class Metrics:
    def __init__(self, cap: int = 4096):
        self.requests_total = 0
        self.errors_total = 0
        self.tokens_generated = 0
        self.in_flight = 0
        self._ttft = collections.deque(maxlen=cap)
        self._lock = threading.Lock()

    def observe_ttft(self, s: float) -> None:
        with self._lock:
            self._ttft.append(s)

    def _quantiles(self, xs):
        if not xs:
            return {"p50": 0.0, "p90": 0.0, "p99": 0.0, "count": 0}
        s = sorted(xs)
        q = lambda f: s[min(len(s) - 1, int(f * (len(s) - 1)))]
        return {"p50": q(0.5), "p90": q(0.9), "p99": q(0.99), "count": len(s)}

    def snapshot(self) -> dict:
        with self._lock:
            tt = list(self._ttft)
        return {"requests_total": self.requests_total, "errors_total": self.errors_total,
                "tokens_generated_total": self.tokens_generated, "in_flight_requests": self.in_flight,
                "ttft_seconds": self._quantiles(tt)}

    def render(self, kv: dict) -> str:
        s = self.snapshot()
        lines = [
            "# HELP bloom_requests_total HTTP requests received.", "# TYPE bloom_requests_total counter",
            f"bloom_requests_total {s['requests_total']}",
            "# HELP bloom_errors_total Requests answered with an error.", "# TYPE bloom_errors_total counter",
            f"bloom_errors_total {s['errors_total']}",
            "# HELP bloom_tokens_generated_total Generated tokens.", "# TYPE bloom_tokens_generated_total counter",
            f"bloom_tokens_generated_total {s['tokens_generated_total']}",
            "# HELP bloom_in_flight_requests Requests being served.", "# TYPE bloom_in_flight_requests gauge",
            f"bloom_in_flight_requests {s['in_flight_requests']}",
            "# HELP bloom_ttft_seconds Time to first token (recent requests).", "# TYPE bloom_ttft_seconds summary",
        ]
        for q in ("p50", "p90", "p99"):
            lines.append(f'bloom_ttft_seconds{{quantile="{q[1:] and "0." + q[1:]}"}} {s["ttft_seconds"][q]}')
        lines.append(f"bloom_ttft_seconds_count {s['ttft_seconds']['count']}")
        for k, v in kv.items():
            lines.append(f"# TYPE bloom_kv_{k} gauge")
            lines.append(f"bloom_kv_{k} {v}")
        return "\n".join(lines) + "\n"
