"""Prometheus text metrics of the server (MLXLMServer/Runtime/ServerMetrics.swift:25-111)
plus the engine's capacity gauges (CBv2CapacitySnapshot)."""
from __future__ import annotations

import threading
import time


class ServerMetrics:
    def __init__(self):
        self.lock = threading.Lock()
        self.start = time.time()
        self.c = {"requests_total": 0, "chat_requests_total": 0, "completion_requests_total": 0,
                  "response_requests_total": 0, "embedding_requests_total": 0, "errors_total": 0,
                  "prompt_tokens_total": 0, "completion_tokens_total": 0, "cached_prompt_tokens_total": 0}

    def inc(self, name, n=1):
        with self.lock:
            self.c[name] = self.c.get(name, 0) + n

    def render(self, engine=None) -> str:
        lines = []
        with self.lock:
            for k, v in self.c.items():
                lines.append(f"# TYPE b200lm_{k} counter")
                lines.append(f"b200lm_{k} {v}")
        lines.append("# TYPE b200lm_uptime_seconds gauge")
        lines.append(f"b200lm_uptime_seconds {time.time() - self.start:.3f}")
        if engine is not None:
            cap = engine.capacity()
            for k in ("active_requests", "waiting_requests", "kv_pages_total", "kv_pages_used", "kv_pages_free",
                      "active_tokens", "steps", "decode_rows"):
                lines.append(f"# TYPE b200lm_engine_{k} gauge")
                lines.append(f"b200lm_engine_{k} {getattr(cap, k)}")
            lines.append(f"b200lm_engine_last_step_ms {cap.last_step_ms:.3f}")
            lines.append(f"b200lm_engine_healthy {1 if cap.healthy else 0}")
        return "\n".join(lines) + "\n"
