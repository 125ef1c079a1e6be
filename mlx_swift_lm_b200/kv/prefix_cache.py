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

Tiers (the reference's snapshot tier and prefix checkpoints,
PrefixCacheV2.swift:69-545): with ``host_blocks`` > 0 a block evicted from
the device is first copied into a pinned host pool (every KV layer group of
its pages) and a later match brings it back into fresh device pages instead
of recomputing it; :meth:`PrefixCache.save` / :meth:`PrefixCache.load` write
every cached block (both tiers) to safetensors files and read them back, so a
restarted server starts with its prefixes warm.
"""
from __future__ import annotations

import collections
import json
import os

import torch

from .paged import PAGE, PagedKVCache, _b200host


class HostTier:
    """Pinned host copies of evicted prefix blocks: per KV layer group a slab
    [layers, blocks * pages_per_block, KVH, 16, D] (K and V), LRU over blocks."""

    def __init__(self, cache: PagedKVCache, max_blocks: int, pages_per_block: int):
        self.cache = cache
        self.ppb = pages_per_block
        pin = cache.device.type == "cuda"
        self.k = [torch.empty((g.shape[0], max_blocks * pages_per_block) + tuple(g.shape[2:]), dtype=g.dtype,
                              pin_memory=pin) for g in cache.gk]
        self.v = [torch.empty_like(t) for t in self.k]
        self.free = list(range(max_blocks))
        self.entries: "collections.OrderedDict[bytes, int]" = collections.OrderedDict()
        self.stores = 0
        self.loads = 0

    def _rows(self, slot):
        return slice(slot * self.ppb, (slot + 1) * self.ppb)

    def store(self, h: bytes, pages: list[int]):
        if h in self.entries:
            self.entries.move_to_end(h)
            return
        if not self.free:
            if not self.entries:
                return
            _, slot = self.entries.popitem(last=False)
            self.free.append(slot)
        slot = self.free.pop()
        idx = torch.tensor(pages, dtype=torch.long, device=self.cache.device)
        for g in range(len(self.k)):
            self.k[g][:, self._rows(slot)].copy_(self.cache.gk[g].index_select(1, idx))
            self.v[g][:, self._rows(slot)].copy_(self.cache.gv[g].index_select(1, idx))
        self.entries[h] = slot
        self.stores += 1

    def load(self, h: bytes, pages: list[int]) -> bool:
        slot = self.entries.get(h)
        if slot is None:
            return False
        self.entries.move_to_end(h)
        idx = torch.tensor(pages, dtype=torch.long, device=self.cache.device)
        for g in range(len(self.k)):
            dev = self.cache.gk[g].device
            self.cache.gk[g].index_copy_(1, idx, self.k[g][:, self._rows(slot)].to(dev, non_blocking=True))
            self.cache.gv[g].index_copy_(1, idx, self.v[g][:, self._rows(slot)].to(dev, non_blocking=True))
        self.loads += 1
        return True

    def block(self, h: bytes):
        """(K, V) host tensors of a stored block, per group."""
        slot = self.entries[h]
        return [t[:, self._rows(slot)] for t in self.k], [t[:, self._rows(slot)] for t in self.v]


class StateSnapshots:
    """Recurrent-state snapshots of hybrid models (linear-attention / SSM
    layers) at prefix block boundaries: the state after a sequence consumed
    blocks 0..b is kept under block b's chain hash, so a later request with
    that prefix adopts the blocks' KV pages and continues from the copied
    state instead of recomputing the prefix (the reference's hybrid prefix
    cache, ContinuousBatchingV2/Prefix/HybridPrefixCache.swift:7). LRU over a
    fixed number of device slots shaped like the recurrent-state pool."""

    def __init__(self, rec, max_snapshots: int):
        self.rec = rec
        L = rec.conv.shape[0]
        self.conv = torch.empty((L, max_snapshots) + tuple(rec.conv.shape[2:]), dtype=rec.conv.dtype,
                                device=rec.conv.device)
        self.ssm = torch.empty((L, max_snapshots) + tuple(rec.ssm.shape[2:]), dtype=rec.ssm.dtype,
                               device=rec.ssm.device)
        self.free = list(range(max_snapshots))
        self.entries: "collections.OrderedDict[bytes, int]" = collections.OrderedDict()
        self.saves = 0
        self.restores = 0

    def save(self, h: bytes, slot: int):
        if h in self.entries:
            self.entries.move_to_end(h)
            return
        if not self.free:
            if not self.entries:
                return
            _, i = self.entries.popitem(last=False)
            self.free.append(i)
        i = self.free.pop()
        self.conv[:, i].copy_(self.rec.conv[:, slot])
        self.ssm[:, i].copy_(self.rec.ssm[:, slot])
        self.entries[h] = i
        self.saves += 1

    def restore(self, h: bytes, slot: int) -> bool:
        i = self.entries.get(h)
        if i is None:
            return False
        self.entries.move_to_end(h)
        self.rec.conv[:, slot].copy_(self.conv[:, i])
        self.rec.ssm[:, slot].copy_(self.ssm[:, i])
        self.restores += 1
        return True


class PrefixCache:
    def __init__(self, cache: PagedKVCache, block_size: int = 256, default_salt: str = "", host_blocks: int = 0,
                 state_snapshots: int = 0):
        assert block_size % PAGE == 0, "block size must be a multiple of the page size"
        self.cache = cache
        self.block = block_size
        self.pages_per_block = block_size // PAGE
        self.salt = default_salt
        self.entries: "collections.OrderedDict[bytes, list[int]]" = collections.OrderedDict()
        self.host = HostTier(cache, host_blocks, self.pages_per_block) if host_blocks > 0 else None
        # hybrid models: a match must end at a block whose recurrent state was kept
        self.states = StateSnapshots(cache.rec, state_snapshots) if cache.rec is not None else None
        if cache.rec is not None and state_snapshots <= 0:
            raise ValueError("a prefix cache over recurrent-state layers needs state_snapshots > 0")
        self.hits = 0
        self.misses = 0
        self.hit_tokens = 0
        self.host_hits = 0

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
        if self.states is not None:
            # the longest cached chain that ends at a block with a state snapshot
            n_ok = 0
            for b, h in enumerate(hashes):
                if h not in self.entries and not (self.host is not None and h in self.host.entries):
                    break
                if h in self.states.entries:
                    n_ok = b + 1
            hashes = hashes[:n_ok]
        pages = []
        chain = set()
        for h in hashes:
            ent = self.entries.get(h)
            if ent is None and self.host is not None and h in self.host.entries:
                ent = self._promote(h, chain)
            chain.add(h)
            if ent is None:
                break
            self.entries.move_to_end(h)
            pages.extend(ent)
        if self.states is not None and pages and len(pages) != len(hashes) * self.pages_per_block:
            pages = []  # a block of the chain could not be brought back: its state has no KV
        if not pages:
            self.misses += 1
            return 0
        self.cache.pool.incref(pages)
        n = len(pages) * PAGE
        st.seq.adopt_prefix(pages, n)
        if self.states is not None:
            st.extra["state_restore"] = hashes[len(pages) // self.pages_per_block - 1]
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

    # ------------------------------------------------------------------ hybrid models
    def snapshot_boundary(self, st) -> int:
        """Token count at which a hybrid request's recurrent state is worth
        keeping: the last full block before the prompt's last token (the
        longest prefix a later identical prompt can reuse); 0 if none."""
        if self.states is None or not st.req.prefix_cache_enabled:
            return 0
        return ((st.num_prompt - 1) // self.block) * self.block

    def after_prefill_chunk(self, st, end: int):
        """Keep the state of a hybrid request whose prefill reached a block
        boundary (its state slot now holds the state after `end` tokens)."""
        if self.states is None or not st.req.prefix_cache_enabled or end <= 0 or end % self.block:
            return
        if end > self.snapshot_boundary(st):
            return
        h = self._hashes(st.all_tokens[:end], st.req.cache_salt)[-1]
        self.states.save(h, st.seq.state_slot)

    def restore_state(self, st):
        """Before a matched hybrid request's first forward: its state slot
        gets the snapshot at the end of the adopted prefix."""
        h = st.extra.pop("state_restore", None)
        if h is not None and not self.states.restore(h, st.seq.state_slot):
            raise RuntimeError("prefix state snapshot evicted between match and first forward")

    def _promote(self, h: bytes, keep=()):
        """Bring a host-tier block back into fresh device pages, evicting
        other least-recently-used device blocks (not those in `keep`) to make
        room; None if the pool still has none."""
        pool = self.cache.pool
        if not pool.can_alloc(self.pages_per_block):
            self.evict(self.pages_per_block - pool.num_free, keep)
        if not pool.can_alloc(self.pages_per_block):
            return None
        pages = list(pool.alloc(self.pages_per_block))
        self.host.load(h, pages)
        self.entries[h] = pages
        self.host_hits += 1
        return pages

    def evict(self, need_pages: int, keep=()) -> int:
        """Free least-recently-used blocks whose pages only the cache holds
        (copied to the host tier first when there is one), except `keep`."""
        freed = 0
        pool = self.cache.pool
        for h in list(self.entries.keys()):
            if freed >= need_pages:
                break
            if h in keep:
                continue
            pages = self.entries[h]
            if all(pool.refcount(p) == 1 for p in pages):
                if self.host is not None:
                    self.host.store(h, pages)
                del self.entries[h]
                freed += pool.decref(pages)
        return freed

    # ------------------------------------------------------------------ checkpoints
    def save(self, path: str, shard_blocks: int = 64):
        """Every cached block (device and host tier) to `path`: shards of
        K / V tensors per block and layer group plus ``index.json`` (hash ->
        shard), with the cache geometry it belongs to."""
        from ..loader.safetensors import save_safetensors

        os.makedirs(path, exist_ok=True)
        blocks = []
        for h, pages in self.entries.items():
            idx = torch.tensor(pages, dtype=torch.long, device=self.cache.device)
            blocks.append((h, [g.index_select(1, idx) for g in self.cache.gk],
                           [g.index_select(1, idx) for g in self.cache.gv]))
        if self.host is not None:
            for h in self.host.entries:
                if h not in self.entries:
                    k, v = self.host.block(h)
                    blocks.append((h, k, v))
        index = {}
        for s0 in range(0, len(blocks), shard_blocks):
            name = f"prefix-{s0 // shard_blocks:05d}.safetensors"
            tens = {}
            for h, ks, vs in blocks[s0:s0 + shard_blocks]:
                for g, (k, v) in enumerate(zip(ks, vs)):
                    tens[f"{h.hex()}.{g}.k"] = k
                    tens[f"{h.hex()}.{g}.v"] = v
                index[h.hex()] = name
            save_safetensors(os.path.join(path, name), tens)
        meta = {"block_size": self.block, "group_shapes": [list(s) for s in self.cache.group_shapes],
                "layers": [int(g.shape[0]) for g in self.cache.gk], "dtype": str(self.cache.gk[0].dtype),
                "blocks": index}
        with open(os.path.join(path, "index.json"), "w") as f:
            json.dump(meta, f)
        return len(blocks)

    def load(self, path: str) -> int:
        """Blocks saved by :meth:`save` into this cache (device pages while the
        pool has room, then the host tier). The geometry must match."""
        from ..loader.safetensors import load_safetensors

        with open(os.path.join(path, "index.json")) as f:
            meta = json.load(f)
        if meta["block_size"] != self.block or meta["group_shapes"] != [list(s) for s in self.cache.group_shapes] \
                or meta["layers"] != [int(g.shape[0]) for g in self.cache.gk]:
            raise ValueError("prefix checkpoint was written for another cache geometry")
        n = 0
        by_shard: dict[str, list[str]] = {}
        for hx, shard in meta["blocks"].items():
            by_shard.setdefault(shard, []).append(hx)
        pool = self.cache.pool
        for shard, hxs in by_shard.items():
            tens, _ = load_safetensors(os.path.join(path, shard))
            for hx in hxs:
                h = bytes.fromhex(hx)
                if h in self.entries:
                    continue
                G = len(self.cache.gk)
                if pool.can_alloc(self.pages_per_block):
                    pages = list(pool.alloc(self.pages_per_block))
                    idx = torch.tensor(pages, dtype=torch.long, device=self.cache.device)
                    for g in range(G):
                        self.cache.gk[g].index_copy_(1, idx, tens[f"{hx}.{g}.k"].to(self.cache.gk[g].device))
                        self.cache.gv[g].index_copy_(1, idx, tens[f"{hx}.{g}.v"].to(self.cache.gv[g].device))
                    self.entries[h] = pages
                elif self.host is not None and self.host.free:
                    slot = self.host.free.pop()
                    for g in range(G):
                        self.host.k[g][:, self.host._rows(slot)].copy_(tens[f"{hx}.{g}.k"])
                        self.host.v[g][:, self.host._rows(slot)].copy_(tens[f"{hx}.{g}.v"])
                    self.host.entries[h] = slot
                else:
                    break
                n += 1
        return n

    def clear(self):
        for pages in self.entries.values():
            self.cache.pool.decref(pages)
        self.entries.clear()

    @property
    def num_blocks(self) -> int:
        return len(self.entries)
