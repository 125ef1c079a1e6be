"""EngineV2: the continuous-batching serving engine.

Public surface mirrors the reference engine (ContinuousBatchingV2/EngineV2.swift:
``init`` :282, ``submit`` :1428, ``cancel`` :1836, ``capacity`` :1842,
``shutdown`` :1922; health :216-224) and its step loop
(EngineLoopV2.swift:3044-3373 ``engineStep``, :5218 ``finalize``).

One step = plan (host scheduler) -> one flattened forward over decode rows and
prefill chunks -> fused sampling -> finalize (commit KV, stop checks,
detokenise, stream events). Pure-decode steps replay a CUDA graph captured for
the batch bucket (:mod:`.graphs`) and, with ``chained_decode``, the next
step's graph is launched on the device-resident sampled tokens of this step
before its tokens are read back, so host finalisation overlaps GPU work (the
reference's chained-decode fast path, EngineLoopV2.swift:3115-3250, 4394).
"""
from __future__ import annotations

import collections
import os
import threading
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from ..kv.paged import PAGE, PagedKVCache
from ..models.batch import ForwardBatch
from ..ops.attention import decode_max_parts
from .detok import IncrementalDetokenizer, StopHoldback
from .graphs import PENDING
from .sampler import Sampler
from .scheduler import Scheduler, SchedulerConfig, Status
from .types import CapacitySnapshot, Event, FinishReason, Request, now

STREAM_CAPACITY = 256  # events buffered per request before backpressure pauses it


NON_FINITE_MESSAGE = "non-finite logits: the model produced NaN or infinity"
_NVTX = os.environ.get("B200LM_NVTX", "0") == "1"


class _nvtx:
    """NVTX range around a phase of a step (no-op unless B200LM_NVTX=1)."""

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        if _NVTX:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if _NVTX:
            torch.cuda.nvtx.range_pop()
        return False


@dataclass
class EngineConfig:
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    kv_tokens: int | None = None  # pool size in tokens (default: enough for max_concurrent * max_model_len)
    kv_bytes: int | None = None
    kv_memory_fraction: float | None = None  # CUDA: size the pool to this fraction of the HBM left after weights
    kv_fp8: bool = False
    max_model_len: int = 8192
    use_cuda_graphs: bool = True
    graph_buckets: tuple = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128)
    chained_decode: bool = True
    enable_prefix_cache: bool = False
    prefix_block_size: int = 256
    prefix_host_blocks: int = 0  # pinned host tier of the prefix cache (blocks of prefix_block_size tokens)
    # hybrid models (recurrent-state layers): device snapshots of the state at prefix block
    # boundaries; a prefix is reused only up to a block with a snapshot (0 = no prefix cache)
    prefix_state_snapshots: int = 16
    # ring storage for sliding-window layers (window + one step of pages per
    # request instead of the whole context); None: on unless prefix caching is
    window_ring: bool | None = None
    step_timeout_s: float = 30.0  # watchdog (background mode)
    admission_timeout_s: float = 0.0  # legacy knobs, folded into `leases` when set
    decode_progress_timeout_s: float = 0.0
    leases: object = None  # engine.leases.LeaseConfig; None = no leases
    clock: object = None  # injectable monotonic clock (tests)
    # (open_id, close_id[, starts_inside]) thought markers for integer Request.reasoning_budget values
    reasoning_markers: tuple | None = None
    admission: object = None  # engine.admission.AdmissionConfig (watermark, auxiliary bytes); None = defaults


class RequestStream:
    """Per-request event stream. Iterating drives the engine when it is not
    running its own background loop."""

    def __init__(self, engine: "EngineV2", st):
        self.engine = engine
        self.st = st
        self.q: collections.deque = collections.deque()
        self.cv = threading.Condition()
        self.done = False

    @property
    def request_id(self) -> int:
        return self.st.req.id

    def put(self, ev: Event):
        with self.cv:
            self.q.append(ev)
            if len(self.q) >= STREAM_CAPACITY and not ev.finished:
                self.st.paused = True
            self.cv.notify_all()

    def get(self, timeout: float | None = None) -> Event | None:
        eng = self.engine
        while True:
            with self.cv:
                if self.q:
                    ev = self.q.popleft()
                    if self.st.paused and len(self.q) < STREAM_CAPACITY // 2:
                        self.st.paused = False
                    return ev
                if eng.background:
                    if not self.cv.wait(timeout):
                        return None
                    continue
            if not eng.step_once_for_stream():
                return None

    def __iter__(self):
        while not self.done:
            ev = self.get()
            if ev is None:
                return
            if ev.finished:
                self.done = True
            yield ev

    async def __aiter__(self):
        import asyncio

        loop = asyncio.get_running_loop()
        while not self.done:
            ev = await loop.run_in_executor(None, self.get, 0.5)
            if ev is None:
                if not self.engine.background and not self.engine.sched.has_work():
                    return
                continue
            if ev.finished:
                self.done = True
            yield ev

    def tokens(self) -> list[int]:
        out = []
        for ev in self:
            out.extend(ev.tokens)
        return out


class EngineV2:
    def __init__(self, model, tokenizer=None, config: EngineConfig | None = None, eos_token_ids=None,
                 graph_runner=None):
        self.model = model
        self.tok = tokenizer
        self.cfg = config or EngineConfig()
        self.device = model.device
        sc = self.cfg.scheduler
        kv_tokens = self.cfg.kv_tokens or sc.max_concurrent_requests * self.cfg.max_model_len
        # recurrent-state slots (hybrid models): every running request holds one
        seqs = sc.max_concurrent_requests
        if self.cfg.kv_memory_fraction and self.device.type == "cuda" and self.cfg.kv_bytes is None:
            from ..kv.memory import kv_budget_bytes

            self.cfg.kv_bytes = kv_budget_bytes(self.device, self.cfg.kv_memory_fraction)
        ring_chunk = self._window_ring_chunk(model)
        if self.cfg.kv_bytes is not None:
            self.kv = PagedKVCache.for_model(model, kv_bytes=self.cfg.kv_bytes, kv_fp8=self.cfg.kv_fp8, max_seqs=seqs,
                                             ring_chunk=ring_chunk, max_len=self.cfg.max_model_len)
        else:
            self.kv = PagedKVCache.for_model(model, max_tokens=kv_tokens, kv_fp8=self.cfg.kv_fp8, max_seqs=seqs,
                                             ring_chunk=ring_chunk, max_len=self.cfg.max_model_len)
        self.prefix_cache = None
        # an overwritten window ring cannot be shared; hybrid models reuse a
        # prefix only up to a block boundary with a recurrent-state snapshot
        if (self.cfg.enable_prefix_cache and not self.kv.ring_pages
                and (self.kv.rec is None or self.cfg.prefix_state_snapshots > 0)):
            from ..kv.prefix_cache import PrefixCache

            self.prefix_cache = PrefixCache(self.kv, self.cfg.prefix_block_size,
                                            host_blocks=self.cfg.prefix_host_blocks,
                                            state_snapshots=self.cfg.prefix_state_snapshots
                                            if self.kv.rec is not None else 0)
        from .admission import AdmissionConfig, AdmissionLedger, layer_kinds_for

        rec_bytes = self.kv.rec.bytes_per_seq if self.kv.rec is not None else 0
        # a ring-storage request holds a fixed number of ring pages whatever its length
        rec_bytes += self.kv.ring_pages * self.kv.ring_page_bytes
        cap = self.kv.num_pages * self.kv.page_bytes + rec_bytes * seqs
        self.ledger = AdmissionLedger(layer_kinds_for(model, self.cfg.kv_fp8), cap,
                                      self.cfg.admission or AdmissionConfig(fixed_bytes_per_request=rec_bytes))
        self.sched = Scheduler(sc, self.kv, self.prefix_cache, self.ledger)
        self.sampler = Sampler(model.cfg.vocab_size, self.device)
        self.eos = set(eos_token_ids or [])
        self.states: dict[int, object] = {}
        self.streams: dict[int, RequestStream] = {}
        self.background = False
        self.healthy = True
        self.on_step_wedge = None
        self.comm_guard = None  # parallel.health.CommGuard of a multi-rank engine
        # steps by kind: decode-graph launches, eager forwards, MTP rounds
        self.step_kinds = {"graph": 0, "eager": 0, "mtp": 0}
        self.steps = 0
        self.last_step_ms = 0.0
        self._lock = threading.RLock()
        self._thread = None
        self._stop = threading.Event()
        self._step_started = None
        self._clock = self.cfg.clock or time.monotonic
        self._lease_cfg = self.cfg.leases
        if self._lease_cfg is None and (self.cfg.admission_timeout_s > 0 or self.cfg.decode_progress_timeout_s > 0):
            from .leases import LeaseConfig

            self._lease_cfg = LeaseConfig(admission_s=self.cfg.admission_timeout_s, prefill_s=0.0,
                                          decode_s=self.cfg.decode_progress_timeout_s, backpressure_s=0.0,
                                          decode_floor_tps=0.0)
        self.max_pages = PagedKVCache.pages_for(self.cfg.max_model_len)
        self.graphs = graph_runner
        if (self.graphs is None and self.device.type == "cuda" and self.cfg.use_cuda_graphs
                and getattr(model, "pp_stages", 1) == 1):
            from .graphs import DecodeGraphRunner  # noqa: F811

            self.graphs = DecodeGraphRunner(self)
        self._inflight = None  # chained decode: (plan rows, device tokens, event)
        self.mtp = None  # MTPDriver when speculative decoding is enabled
        self.h2d_bytes = 0  # eager-path step inputs copied host -> device
        self.d2h_bytes = 0  # eager-path sampled tokens read back
        self.forward_shapes: list[tuple[int, int]] = []
        self.non_finite_rows = 0  # rows ended because their logits held NaN / infinity
        self.record_shapes = False
        from .diagnostics import Diagnostics

        d = Diagnostics()
        self.diagnostics = d if d.profile else None  # opt-in (B200LM_STEP_PROFILE=1 or assign one)

    def _window_ring_chunk(self, model) -> int:
        """Tokens one step may write for a sequence when sliding-window layers
        get ring storage, else 0. Ring storage is on by default where it
        applies (``EngineConfig.window_ring`` None), and off with prefix
        caching (ring pages are overwritten, so they cannot be shared) or for
        models whose forward does not route per-layer tables."""
        on = self.cfg.window_ring
        if on is None:
            on = not self.cfg.enable_prefix_cache
        if not on or not getattr(model, "supports_window_ring", False):
            return 0
        if model.tp.world != 1 or getattr(model, "pp_stages", 1) != 1:
            return 0
        sc = self.cfg.scheduler
        return max(sc.prefill_chunk_size, 1) + 1

    def enable_mtp(self, module, config=None):
        """Speculative decoding with an MTP draft module (greedy rows)."""
        from .mtp import MTPDriver

        if self.kv.rec is not None:
            raise ValueError("MTP rollback needs per-position recurrent states; hybrid models decode without MTP")
        if self.kv.ring_pages:
            raise ValueError("MTP verification does not route ring-storage page tables; build the engine with "
                             "EngineConfig(window_ring=False)")

        self.mtp = MTPDriver(self, module, config)
        # the draft module's own paged KV is per-token auxiliary memory of every request
        mk = self.mtp.kv
        self.ledger.cfg.auxiliary_bytes_per_token = mk.page_bytes // 16
        self.ledger.update_capacity(self.ledger.capacity_bytes + mk.num_pages * mk.page_bytes)
        return self.mtp

    # ------------------------------------------------------------------ submit / cancel
    def submit(self, req: Request) -> RequestStream:
        total = len(req.prompt_tokens) + req.max_tokens
        if not req.prompt_tokens:
            raise ValueError("empty prompt")
        if total > self.cfg.max_model_len:
            raise ValueError(f"prompt + max_tokens = {total} exceeds max_model_len {self.cfg.max_model_len}")
        if not self.sched.can_ever_fit(total):
            raise ValueError("request can never fit in the KV pool")
        if req.mm is not None:
            # placeholder token ids do not identify the image: no prefix reuse;
            # MTP drafts from text positions only
            req.prefix_cache_enabled = False
            sc = self.cfg.scheduler
            if req.mm.get("prefix_lm") and len(req.prompt_tokens) > min(sc.prefill_chunk_size,
                                                                         sc.max_batched_tokens_per_step):
                raise ValueError(f"a prefix-LM prompt of {len(req.prompt_tokens)} tokens is prefilled in one chunk: "
                                 f"raise prefill_chunk_size / max_batched_tokens_per_step")
        lora_slot = -1
        if req.lora is not None:
            bl = getattr(self.model, "batched_lora", None)
            if bl is None:
                raise ValueError(f"request names adapter {req.lora!r} but the model serves no batched adapters "
                                 "(attach adapters.batched.BatchedLoRA, or merge the adapter)")
            lora_slot = bl.slot(req.lora)
        from .reasoning import ReasoningBudgetState, resolve_budget

        budget = resolve_budget(req.reasoning_budget, self.cfg.reasoning_markers)
        with self._lock:
            ftd = req.first_token_deadline
            if ftd is not None:
                from .leases import TerminalCause, project_first_token_s

                c = self._clock()
                if c + project_first_token_s(self.sched, len(req.prompt_tokens), ftd, req.priority) > ftd.deadline:
                    return self._rejected(req, TerminalCause.FIRST_TOKEN_DEADLINE)
            st = self.sched.add(req)
            st.timing.submitted = now()
            st.extra["submit_clock"] = self._clock()
            if self._lease_cfg is not None:
                from .leases import RequestLeases

                st.extra["lease"] = RequestLeases(st.extra["submit_clock"], self._lease_cfg, len(req.prompt_tokens),
                                                  req.max_tokens)
            if self.tok is not None:
                st.detok = IncrementalDetokenizer(self.tok)
            st.extra["hold"] = StopHoldback(req.stop_strings)
            if lora_slot >= 0:
                st.extra["lora_slot"] = lora_slot
            if budget is not None:
                st.extra["budget"] = ReasoningBudgetState(budget)
            stream = RequestStream(self, st)
            st.stream = stream
            self.states[req.id] = st
            self.streams[req.id] = stream
        return stream

    def cancel(self, request_id: int) -> bool:
        with self._lock:
            st = self.states.get(request_id)
            if st is None or st.status == Status.FINISHED:
                return False
            self._drain_inflight()
            self._finish(st, FinishReason.CANCELLED)
            return True

    # ------------------------------------------------------------------ batch build
    def _build_batch(self, plan, dev):
        rows = plan.rows
        nd = sum(1 for r in rows if r.is_decode)
        ids, pos, slots = [], [], []
        for r in rows:
            st = r.state
            toks = st.all_tokens[r.start:r.start + r.num_tokens]
            ids.extend(toks)
            mm = st.req.mm
            if mm is None:
                pos.extend(range(r.start, r.start + r.num_tokens))
            else:  # generated tokens of a multimodal prompt continue at p + delta (M-RoPE)
                pos.extend(p + (mm["delta"] if p >= mm["prompt_len"] else 0)
                           for p in range(r.start, r.start + r.num_tokens))
            slots.extend(st.seq.slots(r.start, r.num_tokens))
        T = len(ids)
        fb = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.int32), positions=torch.tensor(pos, dtype=torch.int32),
                          slots=torch.tensor(slots, dtype=torch.int64), num_decode=nd)
        maxp = max(len(r.state.seq.pages) for r in rows)
        if self.kv.ring_pages:  # sliding-window ring layers: their own slots and logical page tables
            fb.ring_slots = torch.tensor([s for r in rows for s in r.state.seq.ring_slots(r.start, r.num_tokens)],
                                         dtype=torch.int64)
            tabs = [r.state.seq.ring_table(maxp) for r in rows]
            if nd:
                fb.ring_dec_page_table = torch.from_numpy(np.stack(tabs[:nd]))
            if len(rows) > nd:
                fb.ring_pf_page_table = torch.from_numpy(np.stack(tabs[nd:]))
        logit_idx = []
        off = 0
        for r in rows:
            off += r.num_tokens
            if r.sample:
                logit_idx.append(off - 1)
        if nd:
            pt = np.zeros((nd, maxp), np.int32)
            sl = np.zeros(nd, np.int32)
            for i, r in enumerate(rows[:nd]):
                pg = r.state.seq.pages
                pt[i, :len(pg)] = pg
                sl[i] = r.start + 1
            fb.dec_page_table = torch.from_numpy(pt)
            fb.dec_seq_lens = torch.from_numpy(sl)
            fb.dec_max_parts = decode_max_parts(int(sl.max()))
        pf = rows[nd:]
        if pf:
            cu = [0]
            p0 = []
            pt = np.zeros((len(pf), maxp), np.int32)
            for i, r in enumerate(pf):
                cu.append(cu[-1] + r.num_tokens)
                p0.append(r.start)
                pg = r.state.seq.pages
                pt[i, :len(pg)] = pg
            fb.pf_cu_q = torch.tensor(cu, dtype=torch.int32)
            fb.pf_cu_q_host = cu
            fb.pf_pos0 = torch.tensor(p0, dtype=torch.int32)
            fb.pf_page_table = torch.from_numpy(pt)
        if len(logit_idx) != T:
            fb.logit_idx = torch.tensor(logit_idx, dtype=torch.int64)
            fb.logit_idx_host = logit_idx
        fb.row_ranks = self._row_ranks(rows)
        fb.row_states = [r.state for r in rows]
        fb.pf_pos0_host = [r.start for r in rows[nd:]]
        if self.kv.rec is not None:
            fb.state_slots = torch.tensor([r.state.seq.state_slot for r in rows], dtype=torch.int32)
        if getattr(self.model, "batched_lora", None) is not None and any(
                r.state.extra.get("lora_slot", -1) >= 0 for r in rows):
            fb.lora_slots = torch.tensor([r.state.extra.get("lora_slot", -1) for r in rows
                                          for _ in range(r.num_tokens)], dtype=torch.int32)
        if dev.type == "cuda":
            for name in ("input_ids", "positions", "slots", "dec_page_table", "dec_seq_lens", "pf_cu_q", "pf_pos0",
                         "pf_page_table", "logit_idx", "state_slots", "ring_slots", "ring_dec_page_table",
                         "ring_pf_page_table", "lora_slots"):
                t = getattr(fb, name)
                if t is not None:
                    self.h2d_bytes += t.numel() * t.element_size()
                    setattr(fb, name, t.pin_memory().to(dev, non_blocking=True))
        return fb

    def _row_ranks(self, rows) -> list[int] | None:
        """Data-parallel owner of each row for models that split a step's rows
        across ranks (``model.dp_world > 1``): a request is pinned, at its
        first step, to the rank with the fewest pinned running requests (ties
        to the lower rank). Every rank schedules the same requests in the same
        order, so every rank computes the same assignment."""
        world = getattr(self.model, "dp_world", 1)
        if world <= 1:
            return None
        load = [0] * world
        for st in self.sched.running:
            d = st.extra.get("dp_rank")
            if d is not None:
                load[d] += 1
        out = []
        for r in rows:
            st = r.state
            d = st.extra.get("dp_rank")
            if d is None:
                d = min(range(world), key=lambda j: (load[j], j))
                st.extra["dp_rank"] = d
                load[d] += 1
            out.append(d)
        return out

    # ------------------------------------------------------------------ step
    def step_once_for_stream(self) -> bool:
        with self._lock:
            if not self.sched.has_work() and self._inflight is None:
                return False
            self.step()
            return True

    def step(self) -> list[Event]:
        """Run one engine step; returns the events it emitted. With
        B200LM_NVTX=1 every step (and its forward / finalize phases) is an
        NVTX range, so a system profiler's timeline shows engine steps."""
        guard = self.comm_guard
        try:
            if _NVTX and self.device.type == "cuda":
                torch.cuda.nvtx.range_push(f"engine.step {self.steps}")
                try:
                    events = self._step()
                finally:
                    torch.cuda.nvtx.range_pop()
            else:
                events = self._step()
        except Exception as e:
            # a failed collective aborts the communicator and ends the live streams
            if guard is not None and guard.on_step_error(e):
                with self._lock:
                    self._inflight = None
                    self._step_started = None
                return []
            raise
        if guard is not None:
            guard.after_step(self.steps)
        return events

    def _step(self) -> list[Event]:
        with self._lock:
            t0 = time.perf_counter()
            self._step_started = t0
            self._process_leases()
            events: list[Event] = []
            plan = self.sched.plan()
            self._handle_preemptions(plan)
            if not plan.rows:
                events += self._drain_inflight()
                self._step_started = None
                return events
            if self.record_shapes:
                self.forward_shapes.append((len(plan.decode_rows), plan.num_tokens))
            if self.mtp is not None and self.mtp.eligible(plan):
                if self._inflight is not None:
                    events += self._drain_inflight()
                    self._step_started = None
                    return events + self.step()
                mev = self.mtp.round(plan)
                if mev is not None:
                    self.step_kinds["mtp"] += 1
                    self.steps += 1
                    self.last_step_ms = (time.perf_counter() - t0) * 1e3
                    self._step_started = None
                    return events + mev
            use_graph = (self.graphs is not None and plan.pure_decode and self.graphs.can_run(plan)
                         and not any(self._row_needs_eager(r.state) for r in plan.rows))
            if use_graph:
                # launch on device-resident tokens of the in-flight step (if any), then
                # optimistically advance: this step's input K/V is written and its output
                # is a placeholder until the step is finalized.
                prev = self._inflight
                if self.mtp is not None:
                    for r in plan.rows:
                        self.mtp.drop(r.state)  # history broken: MTP restarts after an eager step
                self.step_kinds["graph"] += 1
                with _nvtx("decode_graph"):
                    handle = self.graphs.launch(plan, chained_from=prev)
                for r in plan.rows:
                    self.sched.commit(r)
                    r.state.all_tokens.append(PENDING)
                self._inflight = (plan, handle)
                if prev is not None:
                    events += self._finalize_inflight(prev)
                if not self.cfg.chained_decode:
                    events += self._drain_inflight()
            else:
                if self._inflight is not None:
                    # the eager path needs every token on the host: finalize, then re-plan
                    events += self._drain_inflight()
                    self._step_started = None
                    return events + self.step()
                self.step_kinds["eager"] += 1
                fb = self._build_batch(plan, self.device)
                hid = None
                dtok = self.diagnostics.begin_forward(self.device) if self.diagnostics is not None else None
                pc = self.prefix_cache
                if pc is not None and pc.states is not None:
                    for r in plan.rows:
                        if "state_restore" in r.state.extra:
                            pc.restore_state(r.state)
                with _nvtx("forward"):
                    if self.mtp is not None:
                        logits, hid = self.model.forward(fb, self.kv, return_both=True)
                    else:
                        logits = self.model.forward(fb, self.kv)
                if self.diagnostics is not None:
                    self.diagnostics.end_forward(dtok, self.steps, fb, logits)
                if pc is not None and pc.states is not None:
                    for r in plan.rows:
                        if not r.is_decode:
                            pc.after_prefill_chunk(r.state, r.start + r.num_tokens)
                srows = [r for r in plan.rows if r.sample]
                if getattr(self.model, "pp_stages", 1) > 1:
                    toks, lp = self._pp_tokens(logits, srows)
                else:
                    toks, lp = self.sampler.sample(logits, [r.state for r in srows])
                toks_host = toks.cpu().tolist() if toks.numel() else []
                self.d2h_bytes += toks.numel() * toks.element_size()
                bad_rows = set()
                flags = getattr(self.sampler, "last_flags", None)
                if flags is not None and len(toks_host):
                    bad_rows = {i for i, f in enumerate(flags.cpu().tolist()) if f}
                    self.d2h_bytes += flags.numel() * flags.element_size()
                for r in plan.rows:
                    self.sched.commit(r)
                    r.state.timing.prefill_chunks += 0 if r.is_decode else 1
                lps = self.sampler.logprob_entries(lp, toks_host, [r.state for r in srows])
                for i, (r, t, l) in enumerate(zip(srows, toks_host, lps)):
                    if i in bad_rows:
                        events += self._non_finite(r.state)
                        continue
                    events += self._accept_token(r.state, int(t), l)
                    if hid is not None and r.state.status != Status.FINISHED:
                        self.mtp.on_first_token(r.state, hid[i])
            self.steps += 1
            self.last_step_ms = (time.perf_counter() - t0) * 1e3
            self._step_started = None
            return events

    def _pp_tokens(self, logits, srows):
        """Pipeline parallelism: the last stage samples, every stage receives
        the tokens (so all schedulers advance identically)."""
        import torch.distributed as dist

        pp = self.model.pp
        lp = None
        if pp.is_last:
            toks, lp = self.sampler.sample(logits, [r.state for r in srows])
            toks = toks.to(torch.int32).contiguous()
        else:
            toks = torch.empty(len(srows), dtype=torch.int32, device=self.device)
        if len(srows):
            dist.broadcast(toks, src=pp.last, group=pp.group)
        return toks, lp

    def _row_needs_eager(self, st) -> bool:
        """Rows the captured decode graphs cannot serve: logit processing
        (bias, penalties), token masks (grammar, reasoning budget), logprobs.
        Plain temperature / top-k / top-p / min-p sampling runs in the sampled
        graph variant when the model supports it; batched-LoRA rows in the
        LoRA variants."""
        sp = st.req.sampling
        sampled_ok = self.graphs is not None and getattr(self.graphs, "sampling", False)
        return ((not sp.greedy and not sampled_ok) or st.req.token_constraint is not None or sp.logprobs
                or sp.top_logprobs > 0 or sp.needs_processing or "budget" in st.extra
                or (st.req.lora is not None and getattr(self.model, "tp_fused", None) is not None))

    def _finalize_inflight(self, inflight) -> list[Event]:
        plan, handle = inflight
        toks_host, flags = self.graphs.read_tokens(handle, len(plan.rows))
        events = []
        for r, t, bad in zip(plan.rows, toks_host, flags):
            st = r.state
            if st.status == Status.FINISHED:
                # the row finished while this step was in flight; its extra K/V went to
                # pages it already released (stream order makes their reuse safe)
                continue
            if bad:
                events += self._non_finite(st)
                continue
            events += self._accept_token(st, int(t), None, index=r.start + 1)
        return events

    def _non_finite(self, st) -> list[Event]:
        """A row whose logits held NaN or infinity defines no token: it ends
        with an error and commits nothing from that position
        (ContinuousBatchingV2/CBv2NonFiniteLogits.swift:16)."""
        self.non_finite_rows += 1
        return self._finish(st, FinishReason.ERROR, error=NON_FINITE_MESSAGE, cause="non_finite_logits")

    def _drain_inflight(self) -> list[Event]:
        if self._inflight is None:
            return []
        inf, self._inflight = self._inflight, None
        return self._finalize_inflight(inf)

    # ------------------------------------------------------------------ finalize
    def _accept_token(self, st, tok: int, lp, index: int | None = None) -> list[Event]:
        t = now()
        if st.status == Status.FINISHED:
            return []
        if index is None:
            st.all_tokens.append(tok)
        else:
            assert st.all_tokens[index] == PENDING, "finalizing a token that is not pending"
            st.all_tokens[index] = tok
        st.gen_step += 1
        st.usage.completion_tokens += 1
        if not st.timing.first_token:
            st.timing.first_token = t
            if st.req.on_prefill_completed:
                st.req.on_prefill_completed(st.usage)
        st.timing.last_token = t
        st.timing.token_times.append(t)
        st.timing.decode_steps += 1
        st.extra["last_progress"] = self._clock()
        if st.req.token_constraint is not None:
            st.req.token_constraint.commit(tok)
        budget = st.extra.get("budget")
        if budget is not None:
            budget.confirm(tok)
        reason = None
        if (tok in st.req.stop_tokens or (tok in self.eos and not st.req.ignore_eos)):
            reason = FinishReason.STOP
        elif st.num_output >= st.req.max_tokens and PENDING not in st.all_tokens[st.num_prompt:]:
            reason = FinishReason.LENGTH
        elif index is not None and index + 1 - st.num_prompt >= st.req.max_tokens:
            reason = FinishReason.LENGTH
        elif st.req.token_constraint is not None and st.req.token_constraint.is_terminated():
            reason = FinishReason.STOP
        text = ""
        emit_tokens = [tok]
        if st.detok is not None:
            if reason == FinishReason.STOP and (tok in st.req.stop_tokens or tok in self.eos):
                emit_tokens = []
                text = st.detok.flush()
            else:
                text = st.detok.push([tok])
            text, stopped = st.extra["hold"].push(text)
            if stopped and reason is None:
                reason = FinishReason.STOP
        ev = Event(st.req.id, tokens=emit_tokens, text=text, logprobs=[lp] if lp is not None else None)
        events = [ev]
        st.stream.put(ev)
        if budget is not None and budget.failure is not None:
            return events + self._finish(st, FinishReason.ERROR, error=budget.failure)
        if reason is not None:
            events += self._finish(st, reason)
        return events

    def _finish(self, st, reason, error=None, cause=None) -> list[Event]:
        if st.status == Status.FINISHED:
            return []
        tail = ""
        if st.detok is not None and reason != FinishReason.STOP:
            tail = st.extra["hold"].push(st.detok.flush())[0] + st.extra["hold"].flush()
        st.timing.finished = now()
        st.finish_reason = reason
        if self.mtp is not None:
            self.mtp.drop(st)
        if self.prefix_cache is not None and reason in (FinishReason.STOP, FinishReason.LENGTH):
            self.prefix_cache.donate(st)
        self.sched.finish(st)
        st.seq.release()
        ev = Event(st.req.id, tokens=[], text=tail, finished=True, finish_reason=reason, usage=st.usage,
                   timing=st.timing, error=error, cause=cause)
        st.stream.put(ev)
        self.states.pop(st.req.id, None)
        self.streams.pop(st.req.id, None)
        return [ev]

    def _handle_preemptions(self, plan):
        """A preempted request restarts its prefill lease (its admission lease
        is not re-armed)."""
        c = self._clock()
        for st in plan.preempted:
            ls = st.extra.get("lease")
            if ls is not None:
                ls.mark_preempted(c)

    # ------------------------------------------------------------------ leases / watchdog
    def _process_leases(self):
        """Advance every request's leases from its progress counters and end
        the ones whose lease expired (typed cause on the terminal event)."""
        if self._lease_cfg is None:
            return
        from .leases import TerminalCause

        c = self._clock()
        for st in list(self.sched.running) + list(self.sched.waiting):
            ls = st.extra.get("lease")
            if ls is None:
                continue
            running = st in self.sched.running
            if running:
                ls.record_progress(c, st.num_computed, st.num_output)
                if st.paused:
                    ls.mark_paused(c)
                else:
                    ls.mark_resumed(c)
            cause = ls.expired_cause(c, running)
            if cause is not None:
                self._finish(st, FinishReason.DEADLINE, TerminalCause.DIAGNOSTIC[cause], cause=cause)

    def _rejected(self, req, cause: str) -> "RequestStream":
        """A stream that ends at once (request refused at submission)."""
        from .leases import TerminalCause
        from .scheduler import RequestState

        st = RequestState(req=req, seq=None, arrival=0)
        st.status = Status.FINISHED
        stream = RequestStream(self, st)
        st.stream = stream
        stream.put(Event(req.id, finished=True, finish_reason=FinishReason.DEADLINE, usage=st.usage,
                         timing=st.timing, error=TerminalCause.DIAGNOSTIC[cause], cause=cause))
        return stream

    def _watchdog(self):
        while not self._stop.wait(0.25):
            t = self._step_started
            if t is not None and time.perf_counter() - t > self.cfg.step_timeout_s and self.healthy:
                self.healthy = False
                for st in list(self.states.values()):
                    try:
                        ev = Event(st.req.id, finished=True, finish_reason=FinishReason.WATCHDOG, usage=st.usage,
                                   timing=st.timing, error="engine step exceeded its timeout", cause="watchdog")
                        st.status = Status.FINISHED
                        st.stream.put(ev)
                    except Exception:
                        pass
                if self.on_step_wedge:
                    self.on_step_wedge()

    # ------------------------------------------------------------------ loop control
    def start(self):
        """Run the step loop on a background thread (server mode)."""
        if self._thread is not None:
            return
        self.background = True
        self._stop.clear()

        def loop():
            while not self._stop.is_set():
                if not self.healthy:
                    time.sleep(0.05)
                    continue
                if self.sched.has_work() or self._inflight is not None:
                    try:
                        self.step()
                    except Exception as e:  # engine error: fail live requests, stay up
                        with self._lock:
                            self._inflight = None
                            for st in list(self.states.values()):
                                self._finish(st, FinishReason.ERROR, repr(e))
                else:
                    time.sleep(0.0005)

        self._thread = threading.Thread(target=loop, daemon=True, name="engine-loop")
        self._thread.start()
        self._wd = threading.Thread(target=self._watchdog, daemon=True, name="engine-watchdog")
        self._wd.start()

    def shutdown(self, timeout: float = 10.0):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None
        with self._lock:
            self._drain_inflight()
            for st in list(self.states.values()):
                self._finish(st, FinishReason.CANCELLED, "engine shutdown")
        self.background = False

    def release_graphs(self):
        """Drop the captured decode graphs and their memory pool. Graphs that
        hold collective calls must go before the process group is destroyed,
        or the exit waits on them."""
        if self.graphs is not None and hasattr(self.graphs, "graphs"):
            self.graphs.graphs.clear()
            getattr(self.graphs, "sgraphs", {}).clear()
            self.graphs.pool = None
        if self.device.type == "cuda":
            import gc

            gc.collect()
            torch.cuda.synchronize(self.device)

    def run_until_idle(self, max_steps: int = 1 << 30) -> list[Event]:
        events = []
        n = 0
        while (self.sched.has_work() or self._inflight is not None) and n < max_steps:
            events += self.step()
            n += 1
        events += self._drain_inflight()
        return events

    # ------------------------------------------------------------------ introspection
    def capacity(self) -> CapacitySnapshot:
        pool = self.kv.pool
        return CapacitySnapshot(active_requests=len(self.sched.running), waiting_requests=len(self.sched.waiting),
                                kv_pages_total=self.kv.num_pages, kv_pages_used=pool.num_used,
                                kv_pages_free=pool.num_free, kv_bytes_per_page=self.kv.page_bytes,
                                active_tokens=sum(s.num_computed for s in self.sched.running), steps=self.steps,
                                last_step_ms=self.last_step_ms, decode_rows=sum(1 for s in self.sched.running
                                                                                if s.is_decode),
                                healthy=self.healthy, ledger_bytes_capacity=self.ledger.capacity_bytes,
                                ledger_bytes_reserved=self.ledger.reserved_bytes + self.ledger.snapshot().external_bytes,
                                admission_watermark_bytes=self.ledger.watermark_bytes)

    # ------------------------------------------------------------------ convenience
    def generate(self, prompts: list[list[int]], max_tokens: int = 64, sampling=None, **kw) -> list[list[int]]:
        from .types import SamplingParams

        sampling = sampling or SamplingParams(temperature=0.0)
        streams = [self.submit(Request(prompt_tokens=list(p), max_tokens=max_tokens, sampling=sampling, **kw))
                   for p in prompts]
        self.run_until_idle()
        out = []
        for s in streams:
            toks = []
            while s.q:
                ev = s.q.popleft()
                toks.extend(ev.tokens)
            out.append(toks)
        return out

    def teacher_forced_top1(self, tokens: list[int]) -> list[int]:
        """Greedy next-token prediction at every position of `tokens` (one prefill)."""
        st = self.sched.add(Request(prompt_tokens=list(tokens), max_tokens=1))
        self.sched.waiting.remove(st)
        try:
            if not st.seq.ensure(len(tokens)):
                raise RuntimeError("no KV capacity")
            slots = st.seq.slots(0, len(tokens))
            dev = self.device
            pt = torch.tensor([st.seq.pages], dtype=torch.int32)
            fb = ForwardBatch(input_ids=torch.tensor(tokens, dtype=torch.int32).to(dev),
                              positions=torch.arange(len(tokens), dtype=torch.int32).to(dev),
                              slots=torch.tensor(slots, dtype=torch.int64).to(dev), num_decode=0,
                              pf_cu_q=torch.tensor([0, len(tokens)], dtype=torch.int32).to(dev),
                              pf_cu_q_host=[0, len(tokens)], pf_pos0=torch.tensor([0], dtype=torch.int32).to(dev),
                              pf_page_table=pt.to(dev))
            if self.kv.rec is not None:
                fb.state_slots = torch.tensor([st.seq.state_slot], dtype=torch.int32).to(dev)
            if self.kv.ring_pages:
                if len(tokens) > self.kv.ring_pages * 16 - self.model.cfg.max_window():
                    raise ValueError("a one-shot prefill longer than the window ring; use window_ring=False")
                fb.ring_slots = torch.tensor(st.seq.ring_slots(0, len(tokens)), dtype=torch.int64).to(dev)
                fb.ring_pf_page_table = torch.from_numpy(st.seq.ring_table(len(st.seq.pages))[None]).to(dev)
            logits = self.model.forward(fb, self.kv)
            return logits.argmax(-1).tolist()
        finally:
            st.seq.release()
