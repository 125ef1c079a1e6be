"""Paged KV storage: one device slab per model, host-side page accounting.

* :class:`PagedKVCache` owns the K and V slabs ``[layers, pages, KVH, 16, D]``
  (bf16, or fp8-e4m3 with a per-layer per-KV-head scale) - a single slab
  allocation for the whole model, never per-page buffers, as the reference's
  ``PagedKVPool`` (ContinuousBatchingV2/Paged/PagedKVPool.swift:23-148).
* :class:`SequenceKV` is one request's page list and token count, with
  growth, speculative rollback and release (PagedSequenceKV.swift:37-1072,
  rollback :412, commitSpeculativeWrite :348).

Page accounting runs in the native host pool (``_b200host.PagePool``).
"""
from __future__ import annotations

import sys
import os

import torch

PAGE = 16

_LIBDIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib")
if _LIBDIR not in sys.path:
    sys.path.insert(0, _LIBDIR)
import _b200host  # noqa: E402  (native host runtime)


class PagedKVCache:
    def __init__(self, num_layers: int, num_pages: int, num_kv_heads: int, head_dim: int,
                 dtype=torch.bfloat16, device="cpu", kv_fp8: bool = False):
        self.num_layers = num_layers
        self.num_pages = num_pages
        self.kvh = num_kv_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        self.kv_fp8 = kv_fp8
        sdt = torch.float8_e4m3fn if kv_fp8 else dtype
        shape = (num_layers, num_pages, num_kv_heads, PAGE, head_dim)
        self.k = torch.zeros(shape, dtype=sdt, device=self.device)
        self.v = torch.zeros(shape, dtype=sdt, device=self.device)
        if kv_fp8:
            # per-layer, per-KV-head dequantisation scales (stored = x / scale)
            self.k_scales = torch.ones((num_layers, num_kv_heads), dtype=torch.float32, device=self.device)
            self.v_scales = torch.ones((num_layers, num_kv_heads), dtype=torch.float32, device=self.device)
        else:
            self.k_scales = self.v_scales = None
        self.pool = _b200host.PagePool(num_pages)
        self.page_bytes = 2 * num_layers * num_kv_heads * PAGE * head_dim * self.k.element_size()

    def layer(self, li: int):
        return self.k[li], self.v[li]

    def k_scale(self, li: int):
        return None if self.k_scales is None else self.k_scales[li]

    def v_scale(self, li: int):
        return None if self.v_scales is None else self.v_scales[li]

    def set_fp8_scales(self, k_scales: torch.Tensor, v_scales: torch.Tensor):
        self.k_scales.copy_(k_scales)
        self.v_scales.copy_(v_scales)

    @property
    def free_pages(self) -> int:
        return self.pool.num_free

    @staticmethod
    def pages_for(num_tokens: int) -> int:
        return (num_tokens + PAGE - 1) // PAGE

    @classmethod
    def for_model(cls, model, max_tokens: int | None = None, kv_bytes: int | None = None, kv_fp8=False,
                  device=None):
        """Size the pool by a token budget or a byte budget."""
        dev = device or model.device
        dt = model.dtype
        es = 1 if kv_fp8 else torch.empty((), dtype=dt).element_size()
        per_page = 2 * model.cfg.num_layers * model.KVH * PAGE * model.D * es
        if kv_bytes is not None:
            n = max(1, kv_bytes // per_page)
        else:
            n = cls.pages_for(max_tokens or 4096) + 1
        return cls(model.cfg.num_layers, n, model.KVH, model.D, dt, dev, kv_fp8)


class SequenceKV:
    """One request's KV pages. `num_tokens` = tokens whose K/V are written."""

    def __init__(self, cache: PagedKVCache):
        self.cache = cache
        self.pages: list[int] = []
        self.num_tokens = 0
        self.shared_prefix_pages = 0  # leading pages borrowed from the prefix cache

    def capacity(self) -> int:
        return len(self.pages) * PAGE

    def pages_needed(self, total_tokens: int) -> int:
        return max(0, PagedKVCache.pages_for(total_tokens) - len(self.pages))

    def ensure(self, total_tokens: int) -> bool:
        """Grow to hold `total_tokens`; False if the pool cannot supply pages."""
        need = self.pages_needed(total_tokens)
        if need == 0:
            return True
        if not self.cache.pool.can_alloc(need):
            return False
        self.pages.extend(self.cache.pool.alloc(need))
        return True

    def adopt_prefix(self, pages: list[int], num_tokens: int):
        """Start from shared, already-filled pages (refcounts taken by caller)."""
        assert not self.pages
        self.pages = list(pages)
        self.num_tokens = num_tokens
        self.shared_prefix_pages = len(pages)

    def slot(self, pos: int) -> int:
        return self.pages[pos // PAGE] * PAGE + pos % PAGE

    def slots(self, start: int, n: int) -> list[int]:
        pg = self.pages
        return [pg[p // PAGE] * PAGE + p % PAGE for p in range(start, start + n)]

    def rollback(self, n: int) -> int:
        """Forget the last n written tokens and release pages beyond the new end."""
        n = min(n, self.num_tokens)
        self.num_tokens -= n
        keep = max(self.shared_prefix_pages, PagedKVCache.pages_for(self.num_tokens))
        if keep < len(self.pages):
            extra = self.pages[keep:]
            self.pages = self.pages[:keep]
            self.cache.pool.decref(extra)
        return n

    def release(self):
        if self.pages:
            self.cache.pool.decref(self.pages)
        self.pages = []
        self.num_tokens = 0
        self.shared_prefix_pages = 0
