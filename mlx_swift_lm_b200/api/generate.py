"""Single-request generation API.

Parity: MLXLMCommon/Evaluate.swift -
``GenerateParameters`` (:127-327), ``TokenIterator`` (:905-1207, ``next`` :1159),
``SpeculativeTokenIterator`` (:1239-1715), the ``generate`` family (:1927-2720)
with ``Generation`` chunk / info events and completion info.

``generate`` runs through the continuous-batching engine (one request is a
batch of one; on a GPU this is the CUDA-graph decode path).
``TokenIterator`` is the legacy dense-KV iterator of the reference (one
sequence, concatenating cache), kept for parity and for CPU use; it honours
``max_kv_size`` by keeping a rotating window of the most recent tokens.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from ..engine.types import FinishReason, Request, SamplingParams


@dataclass
class GenerateParameters:
    max_tokens: int | None = 256
    max_kv_size: int | None = None
    temperature: float = 0.6
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    repetition_penalty: float | None = None
    repetition_context_size: int = 20
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    seed: int | None = None
    logit_bias: dict = field(default_factory=dict)
    top_logprobs: int = 0
    prefill_step_size: int = 512
    stop: list[str] = field(default_factory=list)
    kv_bits: int | None = None  # quantized legacy KV (affine 4/8)
    kv_group_size: int = 64
    kv_scheme: str | None = None  # KV compression (kv.compress): affine4/8, turbo<K>v<V>, varn<K>v<V>[t32|t64]

    def sampling(self) -> SamplingParams:
        return SamplingParams(temperature=self.temperature, top_p=self.top_p, top_k=self.top_k, min_p=self.min_p,
                              repetition_penalty=self.repetition_penalty or 1.0,
                              repetition_context_size=self.repetition_context_size,
                              frequency_penalty=self.frequency_penalty, presence_penalty=self.presence_penalty,
                              seed=self.seed, logit_bias=dict(self.logit_bias), top_logprobs=self.top_logprobs,
                              logprobs=self.top_logprobs > 0)


@dataclass
class GenerateCompletionInfo:
    prompt_tokens: int
    generation_tokens: int
    prompt_time: float
    generate_time: float
    stop_reason: str

    @property
    def prompt_tokens_per_second(self) -> float:
        return self.prompt_tokens / self.prompt_time if self.prompt_time > 0 else 0.0

    @property
    def tokens_per_second(self) -> float:
        return self.generation_tokens / self.generate_time if self.generate_time > 0 else 0.0


@dataclass
class Generation:
    """A streamed generation event: a text chunk, a token, or the final info."""
    chunk: str | None = None
    token: int | None = None
    info: GenerateCompletionInfo | None = None
    tool_call: object = None
    reasoning: str | None = None


def generate_stream(engine, prompt_tokens: list[int], params: GenerateParameters | None = None, stop_tokens=(),
                    token_constraint=None, mm=None):
    """Yield :class:`Generation` events for one request through the engine
    (`mm`: the multimodal payload of a vision-language prompt)."""
    params = params or GenerateParameters()
    max_tokens = params.max_tokens or (engine.cfg.max_model_len - len(prompt_tokens))
    req = Request(prompt_tokens=list(prompt_tokens), max_tokens=max_tokens, sampling=params.sampling(),
                  stop_tokens=set(stop_tokens), stop_strings=list(params.stop), token_constraint=token_constraint,
                  mm=mm)
    t0 = time.perf_counter()
    stream = engine.submit(req)
    n = 0
    t_first = None
    reason = FinishReason.STOP
    for ev in stream:
        for tok in ev.tokens:
            if t_first is None:
                t_first = time.perf_counter()
            n += 1
            yield Generation(token=tok)
        if ev.text:
            yield Generation(chunk=ev.text)
        if ev.finished:
            reason = ev.finish_reason
    t1 = time.perf_counter()
    t_first = t_first or t1
    yield Generation(info=GenerateCompletionInfo(len(prompt_tokens), n, t_first - t0, t1 - t_first,
                                                 reason.value if reason else "stop"))


def generate(engine, prompt_tokens: list[int], params: GenerateParameters | None = None, **kw):
    """Blocking generation; returns (tokens, text, info)."""
    toks, text, info = [], [], None
    for g in generate_stream(engine, prompt_tokens, params, **kw):
        if g.token is not None:
            toks.append(g.token)
        if g.chunk:
            text.append(g.chunk)
        if g.info is not None:
            info = g.info
    return toks, "".join(text), info


class TokenIterator:
    """Legacy single-sequence iterator over a dense KV cache.

    Each ``next()`` returns the next token id. Prefill runs in
    ``prefill_step_size`` chunks; ``max_kv_size`` selects a rotating window
    cache (the first tokens kept, as the reference's RotatingKVCache) and
    ``kv_bits`` an affine-quantised cache (:mod:`..kv.legacy`)."""

    def __init__(self, model, prompt_tokens, params: GenerateParameters | None = None, cache=None):
        from ..engine.sampler import row_key
        from ..ops import reference as ref

        from ..kv.legacy import QuantizedKVCache, RotatingKVCache

        self.model = model
        self.params = params or GenerateParameters()
        p = self.params
        if cache is None:
            if p.kv_scheme:
                from ..kv.compress import CompressedKVCache

                cache = CompressedKVCache(model.cfg.num_layers, p.kv_scheme)
            elif p.max_kv_size:
                cache = RotatingKVCache(model.cfg.num_layers, p.max_kv_size)
            elif p.kv_bits:
                cache = QuantizedKVCache(model.cfg.num_layers, p.kv_bits, p.kv_group_size)
            else:
                cache = model.new_cache()
        self.cache = cache
        self.tokens = list(prompt_tokens)
        self.n_generated = 0
        self._ref = ref
        self._row_key = row_key
        toks = torch.tensor(self.tokens, dtype=torch.int64, device=model.device)
        step = self.params.prefill_step_size
        logits = None
        for i in range(0, len(toks), step):
            logits = model.forward_dense(toks[i:i + step], self.cache)
        self._logits = logits[-1]

    def _sample(self, logits):
        p = self.params
        sp = p.sampling()
        rep = self.tokens[-sp.repetition_context_size:] if sp.repetition_penalty != 1.0 else None
        outs = self.tokens[len(self.tokens) - self.n_generated:] if (sp.frequency_penalty or sp.presence_penalty) else None
        lg = self._ref.process_logits_ref(logits.float().cpu(), sp.logit_bias, rep, sp.repetition_penalty, outs,
                                          sp.frequency_penalty, sp.presence_penalty)
        key = self._ref.mix_key(sp.seed if sp.seed is not None else 0x5EED, 0)
        return self._ref.sample_ref(lg, sp.temperature, sp.top_k, sp.top_p, sp.min_p, key, self.n_generated)

    def __iter__(self):
        return self

    def __next__(self) -> int:
        if self.params.max_tokens is not None and self.n_generated >= self.params.max_tokens:
            raise StopIteration
        tok = self._sample(self._logits)
        self.tokens.append(tok)
        self.n_generated += 1
        self._logits = self.model.forward_dense(torch.tensor([tok], device=self.model.device), self.cache)[-1]
        return tok


class SpeculativeTokenIterator:
    """Single-sequence speculative decoding with a draft model over dense KV
    caches (parity: Evaluate.swift:1239-1715).

    Each round the draft model proposes `num_draft` tokens greedily; the
    target scores [last token, drafts] in one forward; drafts are accepted
    while they equal the target's greedy token, then the target's own token
    follows; both caches are trimmed back past the rejected positions.
    Greedy (temperature 0) verification, so the output equals plain greedy
    decoding of the target."""

    def __init__(self, model, draft_model, prompt_tokens, params: GenerateParameters | None = None,
                 num_draft: int = 2):
        self.model, self.draft = model, draft_model
        self.params = params or GenerateParameters(temperature=0.0)
        self.k = num_draft
        self.cache, self.dcache = model.new_cache(), draft_model.new_cache()
        self.tokens = list(prompt_tokens)
        self.n_generated = 0
        self.drafted = self.accepted = 0
        self._pending: list[int] = []
        dev = model.device
        toks = torch.tensor(self.tokens[:-1], dtype=torch.int64, device=dev)
        if len(toks):  # both caches hold every token but the last
            model.forward_dense(toks, self.cache)
            draft_model.forward_dense(toks.to(draft_model.device), self.dcache)
        self._last = self.tokens[-1]

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    def __iter__(self):
        return self

    def _round(self):
        dev, ddev = self.model.device, self.draft.device
        drafts, t = [], self._last
        for _ in range(self.k):
            lg = self.draft.forward_dense(torch.tensor([t], device=ddev), self.dcache)[-1]
            t = int(lg.argmax())
            drafts.append(t)
        seq = [self._last] + drafts
        lg = self.model.forward_dense(torch.tensor(seq, device=dev), self.cache)
        pred = lg.argmax(-1).tolist()  # target token after each position
        a = 0
        while a < self.k and drafts[a] == pred[a]:
            a += 1
        self.drafted += self.k
        self.accepted += a
        emit = drafts[:a] + [pred[a]]
        # caches hold [last, d1..dk]; keep last + accepted drafts
        self.cache.trim(self.k - a)
        self.dcache.trim(max(0, self.dcache.offset - self.cache.offset))
        if a == self.k:  # the draft cache lacks the last accepted draft
            self.draft.forward_dense(torch.tensor([drafts[-1]], device=ddev), self.dcache)
        self._last = emit[-1]
        return emit

    def __next__(self) -> int:
        if self.params.max_tokens is not None and self.n_generated >= self.params.max_tokens:
            raise StopIteration
        if not self._pending:
            self._pending = self._round()
        tok = self._pending.pop(0)
        self.tokens.append(tok)
        self.n_generated += 1
        return tok


def generate_mtp(engine, prompt_tokens: list[int], params: GenerateParameters | None = None):
    """One request through an engine with MTP speculative decoding enabled
    (parity: MTPSpeculativeTokenIterator.swift:36-805, batch-1 MTP: backbone
    forward, MTP draft head, batched verify). Returns (tokens, text, info,
    telemetry) with the round's draft / acceptance counts."""
    assert engine.mtp is not None, "enable MTP on the engine first (EngineV2.enable_mtp)"
    s0 = engine.mtp.stats
    before = (s0.rounds, s0.drafted, s0.accepted, s0.emitted)
    params = params or GenerateParameters(temperature=0.0)
    toks, text, info = generate(engine, prompt_tokens, params)
    s1 = engine.mtp.stats
    d = [a - b for a, b in zip((s1.rounds, s1.drafted, s1.accepted, s1.emitted), before)]
    tele = {"rounds": d[0], "drafted": d[1], "accepted": d[2], "emitted": d[3],
            "acceptance_rate": d[2] / d[1] if d[1] else 0.0}
    return toks, text, info, tele
