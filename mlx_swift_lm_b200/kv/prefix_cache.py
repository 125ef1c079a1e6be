"""Resident prefix cache: full token blocks of finished requests keep their
KV pages (refcounted) and are handed to new requests with the same prefix.

Keys are the SHA-256 chain over fixed token blocks, with an optional
per-request salt in the first hash (``h_0 = H(salt || block_0)``), as in the
reference's prefix cache (ContinuousBatchingV2/PrefixCacheV2.swift:69-545,
BlockHasher.swift:25-141, resident page sharing
Paged/PrefixBlocks/PagedPrefixBlockIndex.swift:10). A match never covers a
prompt's last token (its logits must be computed), the cache evicts least
recently used blocks whose pages no live request holds, and requests with
``prefix_cache_enabled=False`` neither read nor donate.
"""
from __future__ import annotations

import collections

from .paged import PAGE, PagedKVCache, _b200host


class PrefixCache:
    def __init__(self, cache: PagedKVCache, block_size: int = 256, default_salt: str = ""):
        assert block_size % PAGE == 0, "block size must be a multiple of the page size"
        self.cache = cache
        self.block = block_size
        self.pages_per_block = block_size // PAGE
        self.salt = default_salt
        self.entries: "collections.OrderedDict[bytes, list[int]]" = collections.OrderedDict()
        self.hits = 0
        self.misses = 0
        self.hit_tokens = 0

    def _hashes(self, tokens, salt):
        return _b200host.block_hashes(list(tokens), self.block, salt if salt is not None else self.salt)

    def match_and_adopt(self, st) -> int:
        req = st.req
        if not req.prefix_cache_enabled or st.seq.pages:
            return 0
        toks = st.all_tokens
        usable = (len(toks) - 1) // self.block  # never cover the last token
        if usable <= 0:
            self.misses += 1
            return 0
        hashes = self._hashes(toks[: usable * self.block], req.cache_salt)
        pages = []
        for h in hashes:
            ent = self.entries.get(h)
            if ent is None:
                break
            self.entries.move_to_end(h)
            pages.extend(ent)
        if not pages:
            self.misses += 1
            return 0
        self.cache.pool.incref(pages)
        n = len(pages) * PAGE
        st.seq.adopt_prefix(pages, n)
        st.usage.cached_prompt_tokens = n
        self.hits += 1
        self.hit_tokens += n
        return n

    def donate(self, st):
        """Keep the full computed blocks of a finishing request."""
        if not st.req.prefix_cache_enabled:
            return
        n_blocks = st.seq.num_tokens // self.block
        if n_blocks <= 0:
            return
        toks = st.all_tokens[: n_blocks * self.block]
        hashes = self._hashes(toks, st.req.cache_salt)
        for b, h in enumerate(hashes):
            if h in self.entries:
                self.entries.move_to_end(h)
                continue
            pages = st.seq.pages[b * self.pages_per_block:(b + 1) * self.pages_per_block]
            if len(pages) < self.pages_per_block:
                break
            self.cache.pool.incref(pages)
            self.entries[h] = list(pages)

    def evict(self, need_pages: int) -> int:
        """Free least-recently-used blocks whose pages only the cache holds."""
        freed = 0
        pool = self.cache.pool
        for h in list(self.entries.keys()):
            if freed >= need_pages:
                break
            pages = self.entries[h]
            if all(pool.refcount(p) == 1 for p in pages):
                del self.entries[h]
                freed += pool.decref(pages)
        return freed

    def clear(self):
        for pages in self.entries.values():
            self.cache.pool.decref(pages)
        self.entries.clear()

    @property
    def num_blocks(self) -> int:
        return len(self.entries)
