"""Continuous-batching scheduler (host side, vLLM-V1 style).

Semantics follow the reference's SchedulerV2
(ContinuousBatchingV2/SchedulerV2.swift:200-1181; spec
docs/engine-v2/specs/B-scheduler.md:5-21):
  * running rows are scheduled first; a row whose only uncomputed token is its
    last sampled one is a decode row and takes exactly 1 token;
  * rows still prefilling take chunks of at most ``prefill_chunk_size`` within
    the per-step token budget ``max_batched_tokens_per_step``;
  * waiting requests are admitted by priority, then arrival order (FCFS),
    while the running set is below ``max_concurrent_requests``;
  * when the page pool cannot grow a running row, the lowest-priority,
    youngest running row is preempted: its pages are freed, its tokens kept,
    and it is requeued at the front to recompute (``preemptionVictim`` :1109,
    ``requeueOnCapacity`` :1154);
  * rows can be paused (stream backpressure) and resumed.
The scheduler is a pure function of host state: it never touches the device.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

from ..kv.paged import PagedKVCache, SequenceKV
from .types import Request, RequestTiming, Usage


@dataclass
class SchedulerConfig:
    max_concurrent_requests: int = 64
    max_batched_tokens_per_step: int = 2048
    prefill_chunk_size: int = 512
    max_waiting: int = 4096
    enable_prefix_cache: bool = True
    # when > 0, at most this many prefill tokens join a step that also decodes
    mixed_step_prefill_token_cap: int = 0
    # decode-only steps to run between prefill chunks while rows are decoding
    decode_steps_between_prefill_chunks: int = 0


class Status(enum.Enum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2


@dataclass(eq=False)
class RequestState:
    req: Request
    seq: SequenceKV
    arrival: int
    all_tokens: list[int] = field(default_factory=list)
    num_prompt: int = 0
    status: Status = Status.WAITING
    paused: bool = False
    timing: RequestTiming = field(default_factory=RequestTiming)
    usage: Usage = field(default_factory=Usage)
    # generation step counter (RNG counter for sampling)
    gen_step: int = 0
    finish_reason: object = None
    detok: object = None
    stream: object = None
    extra: dict = field(default_factory=dict)

    @property
    def num_computed(self) -> int:
        return self.seq.num_tokens

    @property
    def num_output(self) -> int:
        return len(self.all_tokens) - self.num_prompt

    @property
    def output_tokens(self) -> list[int]:
        return self.all_tokens[self.num_prompt:]

    @property
    def remaining(self) -> int:
        return len(self.all_tokens) - self.seq.num_tokens

    @property
    def is_decode(self) -> bool:
        return self.remaining == 1 and self.num_output > 0


@dataclass
class ScheduledRow:
    state: RequestState
    start: int  # first position computed this step
    num_tokens: int
    is_decode: bool
    sample: bool  # this row emits a token after the step


@dataclass
class StepPlan:
    rows: list[ScheduledRow]
    preempted: list[RequestState]

    @property
    def decode_rows(self) -> list[ScheduledRow]:
        return [r for r in self.rows if r.is_decode]

    @property
    def prefill_rows(self) -> list[ScheduledRow]:
        return [r for r in self.rows if not r.is_decode]

    @property
    def num_tokens(self) -> int:
        return sum(r.num_tokens for r in self.rows)

    @property
    def pure_decode(self) -> bool:
        return bool(self.rows) and all(r.is_decode for r in self.rows)


class Scheduler:
    def __init__(self, cfg: SchedulerConfig, cache: PagedKVCache, prefix_cache=None, ledger=None):
        self.cfg = cfg
        self.cache = cache
        self.prefix_cache = prefix_cache
        self.ledger = ledger  # engine.admission.AdmissionLedger: byte admission with a watermark
        self.waiting: list[RequestState] = []
        self.running: list[RequestState] = []
        self._arrival = 0
        self._decode_streak = 0

    # ------------------------------------------------------------------ queue
    def add(self, req: Request) -> RequestState:
        if len(self.waiting) >= self.cfg.max_waiting:
            raise RuntimeError("waiting queue full")
        self._arrival += 1
        st = RequestState(req=req, seq=SequenceKV(self.cache), arrival=self._arrival,
                          all_tokens=list(req.prompt_tokens), num_prompt=len(req.prompt_tokens))
        st.usage.prompt_tokens = len(req.prompt_tokens)
        self.waiting.append(st)
        return st

    def remove(self, st: RequestState):
        if st in self.running:
            self.running.remove(st)
        if st in self.waiting:
            self.waiting.remove(st)

    def has_work(self) -> bool:
        return bool(self.running) or bool(self.waiting)

    def can_ever_fit(self, num_tokens: int) -> bool:
        if self.ledger is not None and not self.ledger.can_ever_fit(num_tokens):
            return False
        return PagedKVCache.pages_for(num_tokens) <= self.cache.num_pages

    # ------------------------------------------------------------------ preemption
    def _victim(self, exclude) -> RequestState | None:
        cands = [s for s in self.running if s not in exclude]
        if not cands:
            return None
        return min(cands, key=lambda s: (s.req.priority, -s.arrival))

    def preempt(self, st: RequestState):
        st.seq.release()
        if self.ledger is not None:
            self.ledger.release_all(st.req.id)
        st.status = Status.WAITING
        st.timing.preemptions += 1
        if st in self.running:
            self.running.remove(st)
        self.waiting.insert(0, st)

    def _ensure(self, st: RequestState, total_tokens: int) -> bool:
        """Grow a row's pages; on pool exhaustion first evict unreferenced
        prefix-cache blocks, then report failure (the caller may preempt)."""
        ok = st.seq.ensure(total_tokens)
        if not ok and self.prefix_cache is not None:
            need = st.seq.pages_needed(total_tokens) - self.cache.pool.num_free
            if need > 0 and self.prefix_cache.evict(need) > 0:
                ok = st.seq.ensure(total_tokens)
        if ok and self.ledger is not None:
            self.ledger.reserve(st.req.id, total_tokens)
        return ok

    # ------------------------------------------------------------------ plan
    def _snap_cap(self, st, n: int) -> int:
        """Hybrid models with a prefix cache: a prefill chunk stops at the
        prompt's last full block boundary, so the recurrent state there can be
        kept for later requests with the same prefix."""
        pc = self.prefix_cache
        if pc is None or pc.states is None:
            return n
        b = pc.snapshot_boundary(st)
        if st.num_computed < b < st.num_computed + n:
            return b - st.num_computed
        return n

    def plan(self) -> StepPlan:
        cfg = self.cfg
        budget = cfg.max_batched_tokens_per_step
        rows: list[ScheduledRow] = []
        preempted: list[RequestState] = []
        scheduled = set()

        # 1) running rows: decode first (1 token each), then continuing prefills
        decoding = [s for s in self.running if s.is_decode and not s.paused]
        prefilling = [s for s in self.running if not s.is_decode and not s.paused]
        for st in decoding:
            if budget <= 0:
                break
            if st.num_output >= st.req.max_tokens:
                continue  # its last token is still in flight; finalize ends it
            while not self._ensure(st, st.num_computed + 1):
                # lowest priority, then youngest, among rows not yet scheduled this
                # step - possibly the row itself
                victim = self._victim(scheduled)
                if victim is None:
                    victim = st
                self.preempt(victim)
                preempted.append(victim)
                if victim is st:
                    break
            if st.status != Status.RUNNING:
                continue
            rows.append(ScheduledRow(st, st.num_computed, 1, True, True))
            scheduled.add(st)
            budget -= 1
        n_decode = len(rows)
        prefill_cap = budget
        if n_decode and cfg.mixed_step_prefill_token_cap > 0:
            prefill_cap = min(prefill_cap, cfg.mixed_step_prefill_token_cap)
        if n_decode and cfg.decode_steps_between_prefill_chunks > 0:
            if self._decode_streak < cfg.decode_steps_between_prefill_chunks:
                prefill_cap = 0
        pbudget = prefill_cap
        for st in prefilling:
            if pbudget <= 0:
                break
            if st.status != Status.RUNNING:
                continue
            n = self._snap_cap(st, min(st.remaining, cfg.prefill_chunk_size, pbudget))
            if not self._ensure(st, st.num_computed + n):
                continue
            rows.append(ScheduledRow(st, st.num_computed, n, False, st.num_computed + n == len(st.all_tokens)))
            scheduled.add(st)
            pbudget -= n
        # 2) admit waiting requests
        if pbudget > 0:
            order = sorted(self.waiting, key=lambda s: (-s.req.priority, s.arrival))
            for st in order:
                if pbudget <= 0 or len(self.running) >= cfg.max_concurrent_requests:
                    break
                if st in preempted:
                    continue
                if self.prefix_cache is not None and st.num_computed == 0 and cfg.enable_prefix_cache:
                    self.prefix_cache.match_and_adopt(st)
                n = self._snap_cap(st, min(st.remaining, cfg.prefill_chunk_size, pbudget))
                if n <= 0:
                    continue
                mm = st.req.mm
                if mm is not None and mm.get("prefix_lm") and st.num_computed == 0 and n < min(st.remaining,
                                                                                              mm["prompt_len"]):
                    break  # a prefix-LM prompt attends both ways: it is prefilled in one chunk (FCFS kept)
                if self.ledger is not None and not self.ledger.has_headroom(
                        self.ledger.admission_tokens(st.num_prompt, st.num_computed + n, st.req.max_tokens)):
                    break  # byte ledger above the admission watermark: admit later (FCFS order kept)
                if not self._ensure(st, st.num_computed + n):
                    if st.seq.num_tokens and st.seq.shared_prefix_pages:
                        st.seq.release()
                    break
                self.waiting.remove(st)
                self.running.append(st)
                st.status = Status.RUNNING
                rows.append(ScheduledRow(st, st.num_computed, n, st.remaining == 1 and st.num_output > 0,
                                         st.num_computed + n == len(st.all_tokens)))
                scheduled.add(st)
                pbudget -= n
        if any(not r.is_decode for r in rows):
            self._decode_streak = 0
        else:
            self._decode_streak += 1
        # decode rows first, then prefill rows (flattened-batch layout)
        rows.sort(key=lambda r: 0 if r.is_decode else 1)
        return StepPlan(rows, preempted)

    # ------------------------------------------------------------------ commit
    @staticmethod
    def commit(row: ScheduledRow):
        """Mark the row's scheduled tokens as computed (their K/V are written)."""
        row.state.seq.num_tokens = row.start + row.num_tokens

    def finish(self, st: RequestState):
        if self.ledger is not None:
            self.ledger.release_all(st.req.id)
        st.status = Status.FINISHED
        if st in self.running:
            self.running.remove(st)
        if st in self.waiting:
            self.waiting.remove(st)
