"""Block mask-diffusion engine (Nemotron-Labs-Diffusion style models).

Parity: MLXLLM/Models/NemotronLabsDiffusion.swift (``diffusionGenerate``
:573 - causal prompt prefill, then per block of ``block_length`` mask tokens
up to ``block_length`` bidirectional denoising steps over the block against
the cached prefix; each step commits the masked positions whose confidence
p(argmax) reaches ``threshold`` (the single most confident one when none
does), or with no threshold a fixed per-step count from the even schedule
``_get_num_transfer_tokens``; a block that holds EOS with no mask before it
stops early; a finished block is written into the cache by one causal
forward. ``linearSpecGenerate`` :771 - a bidirectional draft of
[next token, masks...] filled in one shot (or by threshold rounds), a
causal verify of the block, acceptance of the longest prefix on which the
verifier agrees plus one bonus token, and rollback of the rest) and the
native block engine of MLXLMCommon/ContinuousBatchingV2/NativeBlockEngine.swift
(concurrent requests; only committed tokens reach the output).

B200 design: the requests are batched. One engine step runs at most two
forwards over the paged KV pool, each holding every row that is in that
phase: a causal forward (prompt chunks, block commits, linear-spec verifies)
and a bidirectional forward (denoising / drafting blocks; the prefill
attention kernel in bidirectional mode lets each block attend to its whole
chunk and its cached prefix). A block's K/V written by a bidirectional step
lands in the pages at the block's positions and is simply overwritten by
the next step or by the causal commit, so no cache trimming is needed. The
per-position greedy token, its probability and the max logit come from one
fused kernel pass over the logits (``ops.argmax_confidence``); one
device-to-host read per forward feeds the host-side commit policy.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..kv.paged import PagedKVCache, SequenceKV
from ..models.batch import ForwardBatch


@dataclass
class DiffusionRequest:
    prompt_tokens: list[int]
    max_new_tokens: int = 128
    block_length: int | None = None  # default: the model's ``block_size``
    threshold: float | None = 0.9  # None / 0: commit by the even per-step schedule
    mode: str = "diffusion"  # "diffusion" | "linear_spec"
    eos_token_id: int | None = None
    request_id: int = -1


@dataclass
class DiffusionEvent:
    request_id: int
    tokens: list[int]  # newly committed tokens
    finished: bool = False
    finish_reason: str | None = None  # "stop" | "length"
    nfe: int = 0  # forward passes this request has taken part in so far


@dataclass
class DiffusionConfig:
    max_rows: int = 64  # requests stepped together
    max_tokens_per_step: int = 8192  # prompt tokens per causal forward (plus blocks)
    prefill_chunk: int = 2048
    kv_tokens: int = 1 << 16  # KV pool size in tokens


def transfer_schedule(mask_count: int, steps: int) -> list[int]:
    """Tokens to commit at each of `steps` steps: the even split with the
    remainder on the first steps."""
    base, rem = divmod(mask_count, steps)
    return [base + (1 if i < rem else 0) for i in range(steps)]


@dataclass
class _Row:
    req: DiffusionRequest
    seq: SequenceKV
    tokens: list[int]  # prompt + generated (+ the block being refined)
    B: int
    mask: int
    phase: str = "prefill"  # prefill | denoise | commit | draft | verify | done
    computed: int = 0  # tokens whose causal K/V are in the cache
    block_start: int = 0
    step: int = 0
    schedule: list[int] = field(default_factory=list)
    emitted: int = 0  # generated tokens already reported
    nfe: int = 0
    next_token: int = -1  # linear spec: the last accepted token (not yet in the cache)
    block: list[int] = field(default_factory=list)  # linear spec draft block

    @property
    def prompt_len(self) -> int:
        return len(self.req.prompt_tokens)


class BlockDiffusionEngine:
    def __init__(self, model, config: DiffusionConfig | None = None, mask_token_id: int | None = None):
        self.model = model
        self.cfg = config or DiffusionConfig()
        mc = model.cfg
        if any(mc.is_linear(i) for i in range(mc.num_layers)) if mc.layer_types else False:
            raise ValueError("block diffusion needs attention-only models (a recurrent state cannot be rolled back)")
        self.mask = int(mask_token_id if mask_token_id is not None else mc.extra.get("mask_token_id", 100))
        self.default_block = int(mc.extra.get("diffusion_block", 32))
        self.kv = PagedKVCache.for_model(model, max_tokens=self.cfg.kv_tokens)
        self.device = model.device
        self.rows: list[_Row] = []
        self.waiting: list[_Row] = []
        self._ids = itertools.count()
        self.forwards = 0

    # ------------------------------------------------------------------ requests
    def submit(self, req: DiffusionRequest) -> int:
        B = req.block_length or self.default_block
        if req.mode not in ("diffusion", "linear_spec"):
            raise ValueError(f"unknown mode {req.mode!r}")
        if req.mode == "diffusion" and req.max_new_tokens % B:
            raise ValueError("max_new_tokens must be a multiple of the block length")
        if not req.prompt_tokens:
            raise ValueError("empty prompt")
        if req.request_id < 0:
            req.request_id = next(self._ids)
        r = _Row(req, SequenceKV(self.kv), list(req.prompt_tokens), B, self.mask)
        self.waiting.append(r)
        return req.request_id

    @property
    def has_work(self) -> bool:
        return bool(self.rows or self.waiting)

    def _admit(self):
        while self.waiting and len(self.rows) < self.cfg.max_rows:
            r = self.waiting[0]
            need = r.prompt_len + r.req.max_new_tokens + r.B
            if not r.seq.ensure(need):
                if not self.rows:
                    raise RuntimeError("the KV pool cannot hold this request")
                break
            self.waiting.pop(0)
            self.rows.append(r)

    # ------------------------------------------------------------------ forwards
    def _forward(self, chunks, bidirectional: bool, logit_rows):
        """chunks: [(row, start, tokens)]; logit_rows: per chunk None (no
        logits), "last" or "all". Returns host (tok, conf, mx) per chunk."""
        dev = self.device
        ids, pos, slots, cu, p0, lidx = [], [], [], [0], [], []
        maxp = max(len(r.seq.pages) for r, _, _ in chunks)
        pt = np.zeros((len(chunks), maxp), np.int32)
        for i, ((r, start, toks), want) in enumerate(zip(chunks, logit_rows)):
            n = len(toks)
            ids.extend(toks)
            pos.extend(range(start, start + n))
            slots.extend(r.seq.slots(start, n))
            if want == "all":
                lidx.extend(range(cu[-1], cu[-1] + n))
            elif want == "last":
                lidx.append(cu[-1] + n - 1)
            cu.append(cu[-1] + n)
            p0.append(start)
            pt[i, :len(r.seq.pages)] = r.seq.pages
            r.nfe += 1
        i32 = dict(dtype=torch.int32)
        fb = ForwardBatch(input_ids=torch.tensor(ids, **i32).to(dev), positions=torch.tensor(pos, **i32).to(dev),
                          slots=torch.tensor(slots, dtype=torch.int64).to(dev), num_decode=0,
                          pf_cu_q=torch.tensor(cu, **i32).to(dev), pf_cu_q_host=cu,
                          pf_pos0=torch.tensor(p0, **i32).to(dev), pf_page_table=torch.from_numpy(pt).to(dev),
                          bidirectional=bidirectional, pf_pos0_host=p0)
        self.forwards += 1
        if not lidx:
            self.model.forward(fb, self.kv, return_residual=True)
            return [None] * len(chunks)
        fb.logit_idx = torch.tensor(lidx, dtype=torch.int64).to(dev)
        fb.logit_idx_host = lidx
        logits = self.model.forward(fb, self.kv)
        tok, conf, mx = (t.cpu().numpy() for t in ops.argmax_confidence(logits))
        out, o = [], 0
        for (r, start, toks), want in zip(chunks, logit_rows):
            n = len(toks) if want == "all" else (1 if want == "last" else 0)
            out.append((tok[o:o + n], conf[o:o + n], mx[o:o + n]) if n else None)
            o += n
        return out

    # ------------------------------------------------------------------ step
    def step(self) -> list[DiffusionEvent]:
        self._admit()
        events: list[DiffusionEvent] = []
        # causal forward: prompt chunks, block commits, linear-spec verifies
        chunks, want, kinds = [], [], []
        budget = self.cfg.max_tokens_per_step
        for r in self.rows:
            if r.phase == "prefill" and budget > 0:
                n = min(r.prompt_len - r.computed, self.cfg.prefill_chunk, budget)
                last = r.computed + n == r.prompt_len
                chunks.append((r, r.computed, r.tokens[r.computed:r.computed + n]))
                want.append("last" if last and r.req.mode == "linear_spec" else None)
                kinds.append(("prefill", n, last))
                budget -= n
            elif r.phase == "commit":
                chunks.append((r, r.block_start, r.tokens[r.block_start:r.block_start + r.B]))
                want.append(None)
                kinds.append(("commit", r.B, True))
            elif r.phase == "verify":
                chunks.append((r, r.computed, list(r.block)))
                want.append("all")
                kinds.append(("verify", r.B, True))
        if chunks:
            res = self._forward(chunks, False, want)
            for (r, _, _), kind, out in zip(chunks, kinds, res):
                events.extend(self._after_causal(r, kind, out))
        # bidirectional forward: denoising / drafting blocks
        chunks = []
        for r in self.rows:
            if r.phase == "denoise":
                chunks.append((r, r.block_start, r.tokens[r.block_start:r.block_start + r.B]))
            elif r.phase == "draft":
                chunks.append((r, r.computed, list(r.block)))
        if chunks:
            res = self._forward(chunks, True, ["all"] * len(chunks))
            for (r, _, _), out in zip(chunks, res):
                events.extend(self._after_bidir(r, out))
        done = [r for r in self.rows if r.phase == "done"]
        for r in done:
            r.seq.release()
            self.rows.remove(r)
        return events

    # ------------------------------------------------------------------ transitions
    def _start_block(self, r: _Row):
        r.block_start = len(r.tokens)
        r.tokens.extend([r.mask] * r.B)
        r.step = 0
        r.schedule = transfer_schedule(r.B, r.B)
        r.phase = "denoise"

    def _after_causal(self, r: _Row, kind, out) -> list[DiffusionEvent]:
        what, n, last = kind
        if what == "prefill":
            r.computed += n
            if not last:
                return []
            if r.req.mode == "diffusion":
                self._start_block(r)
                return []
            tok = int(out[0][-1])
            r.tokens.append(tok)
            r.next_token = tok
            return self._emit(r, self._eos_in_new(r))
        if what == "commit":
            r.computed = r.block_start + r.B
            self._start_block(r)
            return []
        # verify
        ar = [int(t) for t in out[0]]
        blk = r.block
        acc = 0
        while acc < r.B - 1 and ar[acc] == blk[acc + 1]:
            acc += 1
        acc += 1
        r.computed += acc  # block[0] and the matched drafts are causal entries now
        new = ar[:acc]
        r.tokens.extend(new)
        r.next_token = new[-1]
        gen = len(r.tokens) - r.prompt_len
        if gen >= r.req.max_new_tokens:
            del r.tokens[r.prompt_len + r.req.max_new_tokens:]
        return self._emit(r, self._eos_in_new(r))

    def _after_bidir(self, r: _Row, out) -> list[DiffusionEvent]:
        tok, conf, mx = out
        thr = r.req.threshold
        if r.phase == "draft":
            masked = [i for i in range(r.B) if r.block[i] == r.mask]
            if not thr or thr <= 0:
                for i in masked:
                    r.block[i] = int(tok[i])
            else:
                hit = [i for i in masked if conf[i] >= thr]
                if not hit:
                    hit = [max(masked, key=lambda i: (conf[i], -i))]
                for i in hit:
                    r.block[i] = int(tok[i])
            if r.mask not in r.block:
                r.phase = "verify"
            return []
        s = r.block_start
        masked = [i for i in range(r.B) if r.tokens[s + i] == r.mask]
        if thr and thr > 0:
            commit = [i for i in masked if conf[i] >= thr]
            if not commit:
                commit = [max(masked, key=lambda i: (conf[i], -i))]
        else:
            order = sorted(masked, key=lambda i: (-mx[i], i))
            commit = order[:r.schedule[r.step]]
        for i in commit:
            r.tokens[s + i] = int(tok[i])
        r.step += 1
        blk = r.tokens[s:s + r.B]
        eos = r.req.eos_token_id
        stop = False
        if eos is not None and eos in blk:
            stop = r.mask not in blk[:blk.index(eos)]
        if stop or r.mask not in blk or r.step >= r.B:
            if stop:
                cut = s + blk.index(eos) + 1
                del r.tokens[cut:]
                return self._emit(r, True)
            evs = self._emit(r, False)
            if len(r.tokens) - r.prompt_len >= r.req.max_new_tokens:  # last block: no commit forward needed
                return evs + self._finish(r, "length")
            r.phase = "commit"
            return evs
        return []

    def _eos_in_new(self, r: _Row) -> bool:
        eos = r.req.eos_token_id
        if eos is None:
            return False
        gen = r.tokens[r.prompt_len + r.emitted:]
        if eos in gen:
            del r.tokens[r.prompt_len + r.emitted + gen.index(eos) + 1:]
            return True
        return False

    def _emit(self, r: _Row, stop: bool) -> list[DiffusionEvent]:
        new = r.tokens[r.prompt_len + r.emitted:]
        r.emitted += len(new)
        gen = len(r.tokens) - r.prompt_len
        if stop:
            r.phase = "done"
            return [DiffusionEvent(r.req.request_id, new, True, "stop", r.nfe)]
        if r.req.mode == "linear_spec":
            if gen >= r.req.max_new_tokens:
                r.phase = "done"
                return [DiffusionEvent(r.req.request_id, new, True, "length", r.nfe)]
            r.block = [r.next_token] + [r.mask] * (r.B - 1)
            r.phase = "draft"
        return [DiffusionEvent(r.req.request_id, new, False, None, r.nfe)]

    def _finish(self, r: _Row, reason: str) -> list[DiffusionEvent]:
        r.phase = "done"
        return [DiffusionEvent(r.req.request_id, [], True, reason, r.nfe)]

    # ------------------------------------------------------------------ convenience
    def generate(self, requests: list[DiffusionRequest]) -> list[tuple[list[int], int]]:
        """Run requests to completion; returns (prompt + generated tokens,
        forward passes) per request, in order."""
        ids = [self.submit(q) for q in requests]
        out = {i: list(q.prompt_tokens) for i, q in zip(ids, requests)}
        nfe = {i: 0 for i in ids}
        while self.has_work:
            for ev in self.step():
                out[ev.request_id].extend(ev.tokens)
                nfe[ev.request_id] = ev.nfe
        return [(out[i], nfe[i]) for i in ids]


def diffusion_generate(model, prompt_ids: list[int], max_new_tokens: int, block_length: int | None = None,
                       threshold: float | None = 0.9, eos_token_id: int | None = None, engine=None):
    """One request through the block-diffusion engine: (tokens, nfe)."""
    eng = engine or BlockDiffusionEngine(model, DiffusionConfig(max_rows=1))
    return eng.generate([DiffusionRequest(list(prompt_ids), max_new_tokens, block_length, threshold, "diffusion",
                                          eos_token_id)])[0]


def linear_spec_generate(model, prompt_ids: list[int], max_new_tokens: int = 128, block_length: int | None = None,
                         threshold: float = 0.0, eos_token_id: int | None = None, engine=None):
    """Linear self-speculation (bidirectional draft, causal verify): (tokens, nfe)."""
    eng = engine or BlockDiffusionEngine(model, DiffusionConfig(max_rows=1))
    return eng.generate([DiffusionRequest(list(prompt_ids), max_new_tokens, block_length, threshold, "linear_spec",
                                          eos_token_id)])[0]
