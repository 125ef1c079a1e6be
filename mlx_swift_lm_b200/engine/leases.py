"""Per-request monotonic deadline leases and first-token deadline admission.

Parity: ContinuousBatchingV2/CBv2DeadlineLeases.swift:51-394 and
FirstTokenDeadlineAdmissionV2.swift:34-1204.

Leases (all on the engine's injectable monotonic clock, never wall time):

* admission   - time before a request first begins engine work; ends at
                admission and never re-arms after a preemption;
* prefill     - refreshed whenever the request's computed prompt tokens grow;
* decode      - refreshed whenever it emits a token, so a long generation that
                keeps producing tokens never expires;
* backpressure- bounds how long a request may sit paused because its
                consumer does not read its stream (health-neutral);
* safety      - a request-derived absolute ceiling from enqueue (queue
                allowance + prompt / prefill floor + max_tokens / decode floor
                + one re-prefill + slack) that only catches pathology.

Each expiry carries a typed cause (:class:`TerminalCause`).

First-token deadline admission: a request may carry an absolute first-token
deadline plus conservative prefill / decode rates; at submission the engine
projects the work queued ahead of it (prefill tokens of earlier requests and
its own prompt, and the decode steps of running rows that interleave with
them) and rejects the request at once when the projection cannot meet the
deadline, or when a needed rate is missing (fails closed).
"""
from __future__ import annotations

import math
from dataclasses import dataclass


class TerminalCause:
    ADMISSION_TIMEOUT = "admission_timeout"
    PREFILL_STALL = "prefill_stall"
    DECODE_STALL = "decode_stall"
    SAFETY_DEADLINE = "safety_deadline"
    BACKPRESSURE_TIMEOUT = "backpressure_timeout"
    WATCHDOG = "watchdog"
    FIRST_TOKEN_DEADLINE = "first_token_deadline"

    DIAGNOSTIC = {
        ADMISSION_TIMEOUT: "admission lease expired before engine admission",
        PREFILL_STALL: "prefill made no progress within the prefill lease",
        DECODE_STALL: "decode made no token progress within the decode lease",
        SAFETY_DEADLINE: "request exceeded its absolute safety ceiling",
        BACKPRESSURE_TIMEOUT: "request paused on stream backpressure past the backpressure lease",
        WATCHDOG: "engine step exceeded its timeout",
        FIRST_TOKEN_DEADLINE: "projected first token misses the request's deadline",
    }


@dataclass
class LeaseConfig:
    """Lease lengths in seconds (0 disables that lease)."""
    admission_s: float = 120.0
    prefill_s: float = 120.0
    decode_s: float = 120.0
    backpressure_s: float = 120.0
    # safety ceiling floors: deliberately far below any real rate
    decode_floor_tps: float = 1.0  # 0 disables the ceiling
    prefill_floor_tps: float = 200.0
    preemption_slack_s: float = 60.0
    max_ceiling_s: float = 1e9


def safety_ceiling_s(prompt_tokens: int, max_tokens: int, cfg: LeaseConfig) -> float:
    """Absolute lifetime bound from enqueue: queue allowance, prompt at the
    prefill floor, output at the decode floor, one conservative re-prefill
    after a late preemption and a fixed slack; saturated."""
    pre = max(0, prompt_tokens) / cfg.prefill_floor_tps
    dec = max(0, max_tokens) / max(0.01, cfg.decode_floor_tps)
    return min(max(0.0, cfg.admission_s) + 2 * pre + dec + cfg.preemption_slack_s, cfg.max_ceiling_s)


class RequestLeases:
    """Lease state of one request; every transition takes `now` explicitly."""

    def __init__(self, now: float, cfg: LeaseConfig, prompt_tokens: int, max_tokens: int):
        self.cfg = cfg
        self.admission_deadline = now + cfg.admission_s if cfg.admission_s > 0 else math.inf
        self.admitted = False
        self.phase = "prefill"
        self.progress_deadline = math.inf
        self.backpressure_deadline = None
        self.paused = False
        self.safety_deadline = (now + safety_ceiling_s(prompt_tokens, max_tokens, cfg)
                                if cfg.decode_floor_tps > 0 else math.inf)
        self.last_computed = 0
        self.last_generated = 0

    def _lease(self, phase: str) -> float:
        s = self.cfg.prefill_s if phase == "prefill" else self.cfg.decode_s
        return s if s > 0 else math.inf

    def mark_admitted(self, now: float):
        if self.admitted:
            return
        self.admitted = True
        self.phase = "prefill"
        self.progress_deadline = now + self._lease("prefill")

    def record_progress(self, now: float, computed: int, generated: int):
        if not self.admitted:
            self.mark_admitted(now)
        if generated > self.last_generated:
            self.last_generated, self.last_computed = generated, computed
            self.phase = "decode"
            self.progress_deadline = now + self._lease("decode")
        elif computed > self.last_computed:
            self.last_computed = computed
            self.phase = "prefill"
            self.progress_deadline = now + self._lease("prefill")

    def mark_paused(self, now: float):
        if not self.paused:
            self.paused = True
            s = self.cfg.backpressure_s
            self.backpressure_deadline = now + s if s > 0 else math.inf

    def mark_resumed(self, now: float):
        if self.paused:
            self.paused = False
            self.backpressure_deadline = None
            self.progress_deadline = now + self._lease(self.phase)

    def mark_preempted(self, now: float):
        self.last_computed = 0
        self.phase = "prefill"
        self.progress_deadline = now + self._lease("prefill")

    def expired_cause(self, now: float, running: bool) -> str | None:
        if not self.admitted:
            if now > self.admission_deadline:
                return TerminalCause.ADMISSION_TIMEOUT
            return TerminalCause.SAFETY_DEADLINE if now > self.safety_deadline else None
        if self.paused and self.backpressure_deadline is not None:
            return TerminalCause.BACKPRESSURE_TIMEOUT if now > self.backpressure_deadline else None
        if now > self.safety_deadline:
            return TerminalCause.SAFETY_DEADLINE
        if running and now > self.progress_deadline:
            return TerminalCause.PREFILL_STALL if self.phase == "prefill" else TerminalCause.DECODE_STALL
        return None


@dataclass
class FirstTokenDeadline:
    """Admission policy input: absolute deadline (engine clock) and
    conservative service rates. `decode_batch_rows` > 0 charges decode per
    batch step (one measured step of that many rows, scaled linearly by the
    projected rows) instead of per row."""
    deadline: float
    prefill_tps: float | None = None
    decode_tps: float | None = None
    decode_batch_rows: float = 0.0
    decode_tokens_per_step: float = 1.0


def project_first_token_s(sched, prompt_tokens: int, policy: FirstTokenDeadline, priority: int = 0) -> float:
    """Projected seconds until a new request's first token: the prefill work
    queued ahead of it (waiting requests of higher or equal priority and the
    unfinished prompts of running rows) plus its own prompt at the prefill
    rate, plus the decode steps that interleave with those prefill chunks at
    the decode rate. inf when a needed rate is missing (fail closed)."""
    cfg = sched.cfg
    ahead = sum(s.remaining for s in sched.waiting if s.req.priority >= priority)
    ahead += sum(s.remaining for s in sched.running if not s.is_decode)
    work = ahead + prompt_tokens
    if policy.prefill_tps is None or policy.prefill_tps <= 0:
        return math.inf
    t = work / policy.prefill_tps
    decoding = sum(1 for s in sched.running if s.is_decode)
    if decoding:
        if policy.decode_tps is None or policy.decode_tps <= 0:
            return math.inf
        per_step = max(1, min(cfg.prefill_chunk_size, cfg.max_batched_tokens_per_step - decoding))
        steps = math.ceil(work / per_step)
        if policy.decode_batch_rows >= 1:
            step_s = policy.decode_tokens_per_step / policy.decode_tps * max(1.0, decoding / policy.decode_batch_rows)
        else:
            step_s = decoding / policy.decode_tps
        t += steps * step_s
    return t
