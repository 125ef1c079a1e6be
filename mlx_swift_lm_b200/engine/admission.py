"""Admission ledger: byte accounting of the memory each request will hold.

The page pool is the hard truth (a row either gets its pages or the scheduler
preempts); this ledger is the soft truth that decides whether a *new* request
may start, the reference's AdmissionV2 (ContinuousBatchingV2/AdmissionV2.swift:
153-1851: per-layer-kind KV bytes, fixed and auxiliary bytes, watermark,
``reserve`` / ``unreserve`` / ``hasHeadroom`` / ``canEverFit`` / ``snapshot``).

Bytes a request is charged:
* per token, the KV bytes of every attention layer that owns storage
  (``kv_bytes_per_token``: K + V x KV heads x head dim x element size, summed
  over layer kinds; layers that share another layer's KV own nothing);
* per token, auxiliary bytes (an MTP draft module's own KV), rounded up to
  the auxiliary allocation granularity;
* once per request, fixed bytes (a hybrid model's conv + recurrent state slot).

Tokens are charged in whole pages (the pool's allocation granularity). A new
request is admitted only while the ledger stays below ``capacity x (1 -
watermark)``; rows already running may grow into the watermark (their growth
is checked against the hard pool). ``external`` bytes (graph padding rows,
scratch carved from the same budget) count as reserved.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field

PAGE = 16


@dataclass
class LayerKind:
    """Storage of one group of attention layers."""
    layers: int
    kv_heads: int
    head_dim: int
    element_bytes: int = 2
    window: int = 0  # > 0: sliding window (storage still per token until ring pages exist)
    shared: bool = False  # reuses another layer's KV: owns no storage

    def bytes_per_token(self) -> int:
        if self.shared:
            return 0
        return 2 * self.layers * self.kv_heads * self.head_dim * self.element_bytes


@dataclass
class AdmissionConfig:
    watermark_fraction: float = 0.05
    fixed_bytes_per_request: int = 0
    auxiliary_bytes_per_token: int = 0
    auxiliary_token_granularity: int = 1
    # tokens charged at admission beyond the prompt (the first decode steps'
    # growth), as a fraction of max_tokens; the rest is charged as rows grow
    projected_output_fraction: float = 0.0


@dataclass
class LedgerSnapshot:
    capacity_bytes: int
    reserved_bytes: int
    external_bytes: int
    requests: int
    watermark_bytes: int

    @property
    def free_bytes(self) -> int:
        return self.capacity_bytes - self.reserved_bytes - self.external_bytes


@dataclass
class _Entry:
    tokens: int = 0
    bytes: int = 0


class AdmissionLedger:
    def __init__(self, kinds: list[LayerKind], capacity_bytes: int, config: AdmissionConfig | None = None):
        self.kinds = list(kinds)
        self.cfg = config or AdmissionConfig()
        self.kv_bytes_per_token = sum(k.bytes_per_token() for k in self.kinds)
        self._capacity = int(capacity_bytes)
        self._entries: dict[int, _Entry] = {}
        self._reserved = 0
        self._external = 0
        self._lock = threading.Lock()

    # ------------------------------------------------------------------ sizing
    @staticmethod
    def _round(n: int, g: int) -> int:
        return n if g <= 1 else -(-n // g) * g

    def bytes_for(self, tokens: int) -> int:
        """Bytes charged for `tokens` tokens of one request (page-rounded KV +
        granular auxiliary state), without the fixed part."""
        kv = self._round(tokens, PAGE) * self.kv_bytes_per_token
        aux = self._round(tokens, self.cfg.auxiliary_token_granularity) * self.cfg.auxiliary_bytes_per_token
        return kv + aux

    @property
    def capacity_bytes(self) -> int:
        return self._capacity

    @property
    def watermark_bytes(self) -> int:
        return int(self._capacity * self.cfg.watermark_fraction)

    def update_capacity(self, nbytes: int):
        with self._lock:
            self._capacity = int(nbytes)

    def reserve_external(self, nbytes: int):
        with self._lock:
            self._external += int(nbytes)

    def refund_external(self):
        with self._lock:
            self._external = 0

    # ------------------------------------------------------------------ queries
    def can_ever_fit(self, total_tokens: int) -> bool:
        """Could a request of `total_tokens` (prompt + max output) run alone?"""
        need = self.bytes_for(total_tokens) + self.cfg.fixed_bytes_per_request
        return need <= self._capacity - self._external

    def has_headroom(self, additional_tokens: int, new_request: bool = True) -> bool:
        """Would charging `additional_tokens` more (and, for a new request, its
        fixed bytes) keep the ledger under the admission ceiling?"""
        add = self.bytes_for(additional_tokens) + (self.cfg.fixed_bytes_per_request if new_request else 0)
        ceiling = self._capacity - self._external - (self.watermark_bytes if new_request else 0)
        with self._lock:
            return self._reserved + add <= ceiling

    def admission_tokens(self, prompt_tokens: int, first_chunk: int, max_tokens: int) -> int:
        """Tokens a new request is charged when admitted."""
        return first_chunk + int(max_tokens * self.cfg.projected_output_fraction)

    # ------------------------------------------------------------------ mutation
    def reserve(self, rid: int, tokens: int) -> bool:
        """Grow request `rid`'s charge to cover `tokens` tokens in total
        (monotonic; a first reservation also charges the fixed bytes)."""
        with self._lock:
            e = self._entries.get(rid)
            new = e is None
            if new:
                e = self._entries[rid] = _Entry()
            if tokens <= e.tokens and not new:
                return True
            b = self.bytes_for(max(tokens, e.tokens)) + self.cfg.fixed_bytes_per_request
            self._reserved += b - e.bytes
            e.tokens, e.bytes = max(tokens, e.tokens), b
            return True

    def unreserve(self, rid: int, tokens: int):
        """Shrink request `rid`'s charge to `tokens` tokens (rollback, preemption to 0 tokens)."""
        with self._lock:
            e = self._entries.get(rid)
            if e is None:
                return
            tokens = max(0, tokens)
            b = self.bytes_for(tokens) + self.cfg.fixed_bytes_per_request
            self._reserved += b - e.bytes
            e.tokens, e.bytes = tokens, b

    def release_all(self, rid: int):
        with self._lock:
            e = self._entries.pop(rid, None)
            if e is not None:
                self._reserved -= e.bytes

    # ------------------------------------------------------------------ telemetry
    @property
    def reserved_bytes(self) -> int:
        return self._reserved

    def snapshot(self) -> LedgerSnapshot:
        with self._lock:
            return LedgerSnapshot(self._capacity, self._reserved, self._external, len(self._entries),
                                  self.watermark_bytes)


def layer_kinds_for(model, kv_fp8: bool = False) -> list[LayerKind]:
    """Layer kinds of a :class:`DecoderLM`: the layers that own paged KV,
    grouped by (window, KV heads, head dim); linear-attention, FFN-only and
    KV-sharing layers own none (recurrent state is the fixed per-request part)."""
    import torch

    es = 1 if kv_fp8 else torch.empty((), dtype=model.dtype).element_size()
    groups: dict[tuple, int] = {}
    for kvh, d, w in model.kv_layer_geom():
        key = (w, kvh, d)
        groups[key] = groups.get(key, 0) + 1
    return [LayerKind(n, kvh, d, es, window=w) for (w, kvh, d), n in sorted(groups.items())]


__all__ = ["AdmissionConfig", "AdmissionLedger", "LayerKind", "LedgerSnapshot", "layer_kinds_for", "field"]
