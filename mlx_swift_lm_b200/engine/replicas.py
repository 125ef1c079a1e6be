"""Data parallelism for serving: independent engine replicas behind one router.

The reference runs several engines at provider level (docs/engine-v2/specs/
H-provider.md); here one process can own N replicas (typically one per GPU,
each with the whole model) and :class:`EngineReplicas` presents them to the
server as a single engine: ``submit`` routes a request, ``cancel`` finds its
owner, ``capacity`` sums the replicas.

Routing: requests whose prompts share their first block (``affinity_tokens``
tokens, salted with ``cache_salt``) prefer the replica that served that block
last, so prefix-cache pages are reused; the preference yields to the least
loaded replica when the preferred one is busier by more than ``slack``
requests. Load = running + waiting requests (then reserved ledger bytes).
"""
from __future__ import annotations

import hashlib
import threading
from collections import OrderedDict

from .types import CapacitySnapshot


class EngineReplicas:
    def __init__(self, engines: list, affinity_tokens: int = 256, slack: int = 2, affinity_entries: int = 4096):
        assert engines, "need at least one engine"
        self.engines = list(engines)
        self.affinity_tokens = affinity_tokens
        self.slack = slack
        self._owner: dict[int, int] = {}  # request id -> replica
        self._affinity: OrderedDict[bytes, int] = OrderedDict()
        self._affinity_entries = affinity_entries
        self._lock = threading.Lock()
        self.routed = [0] * len(self.engines)

    # ------------------------------------------------------------------ engine surface
    @property
    def cfg(self):
        return self.engines[0].cfg

    @property
    def background(self) -> bool:
        return all(e.background for e in self.engines)

    @property
    def healthy(self) -> bool:
        return all(e.healthy for e in self.engines)

    def start(self):
        for e in self.engines:
            e.start()

    def shutdown(self, timeout: float = 10.0):
        for e in self.engines:
            e.shutdown(timeout)

    def _load(self, i: int):
        e = self.engines[i]
        s = e.sched
        return (len(s.running) + len(s.waiting), getattr(e.ledger, "reserved_bytes", 0))

    def _key(self, req) -> bytes | None:
        toks = req.prompt_tokens[:self.affinity_tokens]
        if len(toks) < self.affinity_tokens:
            return None
        h = hashlib.sha256((req.cache_salt or "").encode())
        h.update(bytes(str(toks), "ascii"))
        return h.digest()

    def route(self, req) -> int:
        with self._lock:
            loads = [self._load(i) for i in range(len(self.engines))]
            best = min(range(len(loads)), key=lambda i: loads[i])
            key = self._key(req)
            pick = best
            if key is not None and key in self._affinity:
                pref = self._affinity[key]
                if loads[pref][0] <= loads[best][0] + self.slack:
                    pick = pref
                self._affinity.move_to_end(key)
            if key is not None:
                self._affinity[key] = pick
                while len(self._affinity) > self._affinity_entries:
                    self._affinity.popitem(last=False)
            self.routed[pick] += 1
            self._owner[req.id] = pick
            return pick

    def submit(self, req):
        i = self.route(req)
        stream = self.engines[i].submit(req)
        return stream

    def cancel(self, request_id: int) -> bool:
        i = self._owner.pop(request_id, None)
        if i is None:
            return any(e.cancel(request_id) for e in self.engines)
        return self.engines[i].cancel(request_id)

    def step(self):
        """Step every replica once (foreground use and tests)."""
        events = []
        for e in self.engines:
            events += e.step()
        return events

    def run_until_idle(self, max_steps: int = 1 << 30):
        events = []
        for _ in range(max_steps):
            if not any(e.sched.has_work() or e._inflight is not None for e in self.engines):
                break
            events += self.step()
        for e in self.engines:
            events += e._drain_inflight()
        return events

    def capacity(self) -> CapacitySnapshot:
        snaps = [e.capacity() for e in self.engines]
        f = lambda k: sum(getattr(s, k) for s in snaps)  # noqa: E731
        return CapacitySnapshot(active_requests=f("active_requests"), waiting_requests=f("waiting_requests"),
                                kv_pages_total=f("kv_pages_total"), kv_pages_used=f("kv_pages_used"),
                                kv_pages_free=f("kv_pages_free"), kv_bytes_per_page=snaps[0].kv_bytes_per_page,
                                active_tokens=f("active_tokens"), steps=max(s.steps for s in snaps),
                                last_step_ms=max(s.last_step_ms for s in snaps), decode_rows=f("decode_rows"),
                                healthy=all(s.healthy for s in snaps),
                                ledger_bytes_capacity=f("ledger_bytes_capacity"),
                                ledger_bytes_reserved=f("ledger_bytes_reserved"),
                                admission_watermark_bytes=f("admission_watermark_bytes"))
