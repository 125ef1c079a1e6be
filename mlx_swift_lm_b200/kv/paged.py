"""Paged KV storage: one device slab per model, host-side page accounting.

* :class:`PagedKVCache` owns the K and V slabs ``[layers, pages, KVH, 16, D]``
  (bf16, or fp8-e4m3 with a per-layer per-KV-head scale) - one slab
  allocation per layer group, never per-page buffers, as the reference's
  ``PagedKVPool`` (ContinuousBatchingV2/Paged/PagedKVPool.swift:23-148).
  Models whose attention layers differ in KV heads or head dim (Gemma 4:
  sliding layers 256-dim, global layers 512-dim with their own KV-head count)
  get one slab per distinct (KVH, D); the groups are co-indexed - page ``p``
  of a sequence addresses page ``p`` of every group's slab - so a page table,
  a slot and a prefix-cache entry cover every layer at once
  (per-layer-kind geometry: ContinuousBatchingV2/LayerKindDerivation.swift:23-189).
* :class:`SequenceKV` is one request's page list and token count, with
  growth, speculative rollback and release (PagedSequenceKV.swift:37-1072,
  rollback :412, commitSpeculativeWrite :348).

Page accounting runs in the native host pool (``_b200host.PagePool``).

Hybrid models (linear-attention layers) also get a :class:`RecurrentStatePool`
(``cache.rec``): one fixed-size conv + delta-rule state per running sequence
instead of pages (the reference's recurrent-state rows,
ContinuousBatchingV2/RecurrentStateV2.swift:13), owned by the sequence's
:class:`SequenceKV` as ``state_slot``.
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


class RecurrentStatePool:
    """Per-sequence state of the linear-attention layers: conv inputs
    [layers, slots, taps-1, C] (model dtype) and the delta-rule state
    [layers, slots, Hv, Dv, Dk] (fp32). The last slot is scratch for padding
    rows of captured decode graphs."""

    def __init__(self, num_layers: int, max_seqs: int, conv_dim: int, Hv: int, Dv: int, Dk: int, taps: int = 4,
                 dtype=torch.bfloat16, device="cpu"):
        self.num_layers, self.max_seqs = num_layers, max_seqs
        self.conv = torch.zeros(num_layers, max_seqs + 1, taps - 1, conv_dim, dtype=dtype, device=device)
        self.ssm = torch.zeros(num_layers, max_seqs + 1, Hv, Dv, Dk, dtype=torch.float32, device=device)
        self._free = list(range(max_seqs - 1, -1, -1))
        self.scratch = max_seqs

    @property
    def num_free(self) -> int:
        return len(self._free)

    def alloc(self) -> int | None:
        return self._free.pop() if self._free else None

    def release(self, slot: int):
        if 0 <= slot < self.max_seqs:
            self._free.append(slot)

    def layer(self, i: int):
        return self.conv[i], self.ssm[i]

    @property
    def bytes_per_seq(self) -> int:
        return (self.conv[:, 0].numel() * self.conv.element_size() + self.ssm[:, 0].numel() * 4)


class PagedKVCache:
    def __init__(self, num_layers: int, num_pages: int, num_kv_heads: int, head_dim: int,
                 dtype=torch.bfloat16, device="cpu", kv_fp8: bool = False, layer_shapes=None,
                 layer_ring=None, ring_pages: int = 0, ring_seqs: int = 0):
        """`layer_shapes`: optional (KVH, D) of every KV layer; layers of one
        shape share a slab. Default: every layer (num_kv_heads, head_dim).

        `layer_ring` (bool per KV layer) with `ring_pages` R > 0: those
        (sliding-window) layers keep a ring of R pages per sequence instead
        of one page per 16 tokens - position p lives on ring page
        (p // 16) % R - drawn from a pool of its own sized for `ring_seqs`
        sequences. R must cover the window plus the longest chunk one step
        writes (WindowedSequenceKV.swift:1-80 stores a window ring per
        sequence; PagedLayerCache.swift:597-616 sizes ring pages)."""
        shapes = [tuple(x) for x in layer_shapes] if layer_shapes else [(num_kv_heads, head_dim)] * num_layers
        ring = [bool(x) for x in layer_ring] if (layer_ring and ring_pages > 0) else [False] * len(shapes)
        self.num_layers = len(shapes)
        self.num_pages = num_pages
        self.device = torch.device(device)
        self.kv_fp8 = kv_fp8
        self.ring_pages = ring_pages if any(ring) else 0
        self.ring_num_pages = ring_seqs * self.ring_pages + 1 if self.ring_pages else 0
        sdt = torch.float8_e4m3fn if kv_fp8 else dtype
        # group g: layers of one (shape, ring) key; _where[li] = (g, index within the group)
        self.group_shapes: list[tuple[int, int]] = []
        self.group_ring: list[bool] = []
        self._where: list[tuple[int, int]] = []
        keys: list[tuple] = []
        counts: dict[tuple, int] = {}
        for sh, rg in zip(shapes, ring):
            key = (sh, rg)
            if key not in counts:
                counts[key] = 0
                keys.append(key)
                self.group_shapes.append(sh)
                self.group_ring.append(rg)
            self._where.append((keys.index(key), counts[key]))
            counts[key] += 1
        self.gk, self.gv = [], []
        for key in keys:
            (kvh, d), rg = key
            shape = (counts[key], self.ring_num_pages if rg else num_pages, kvh, PAGE, d)
            self.gk.append(torch.zeros(shape, dtype=sdt, device=self.device))
            self.gv.append(torch.zeros(shape, dtype=sdt, device=self.device))
        # the first group's slabs and geometry (single-group models: the whole cache)
        self.k, self.v = self.gk[0], self.gv[0]
        self.kvh, self.head_dim = self.group_shapes[0]
        self.layer_shapes = shapes
        self.layer_ring = ring
        kvh_max = max(k for k, _ in shapes)
        if kv_fp8:
            # per-layer, per-KV-head dequantisation scales (stored = x / scale)
            self.k_scales = torch.ones((self.num_layers, kvh_max), dtype=torch.float32, device=self.device)
            self.v_scales = torch.ones((self.num_layers, kvh_max), dtype=torch.float32, device=self.device)
        else:
            self.k_scales = self.v_scales = None
        self.pool = _b200host.PagePool(num_pages)
        self.ring_pool = _b200host.PagePool(self.ring_num_pages) if self.ring_pages else None
        es = self.k.element_size()
        # bytes per page of the growing (per-token) layers; ring layers: bytes per ring page
        self.page_bytes = sum(2 * kvh * PAGE * d * es for (kvh, d), rg in zip(shapes, ring) if not rg)
        self.ring_page_bytes = sum(2 * kvh * PAGE * d * es for (kvh, d), rg in zip(shapes, ring) if rg)
        self.rec: RecurrentStatePool | None = None

    def is_ring(self, li: int) -> bool:
        return self.layer_ring[li]

    @property
    def slab_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.gk + self.gv)

    def layer(self, li: int):
        g, j = self._where[li]
        return self.gk[g][j], self.gv[g][j]

    def k_scale(self, li: int):
        return None if self.k_scales is None else self.k_scales[li, :self.layer_shapes[li][0]]

    def v_scale(self, li: int):
        return None if self.v_scales is None else self.v_scales[li, :self.layer_shapes[li][0]]

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
                  device=None, max_seqs: int = 64, ring_chunk: int = 0, max_len: int | None = None):
        """Size the pool by a token budget or a byte budget. Only attention
        layers hold pages; linear-attention layers get `max_seqs` state slots.
        `ring_chunk` > 0 (the most tokens one step writes for a sequence)
        gives sliding-window layers ring storage for `max_seqs` sequences
        (carved from `kv_bytes` first)."""
        dev = device or model.device
        dt = model.dtype
        es = 1 if kv_fp8 else torch.empty((), dtype=dt).element_size()
        geom = model.kv_layer_geom() if hasattr(model, "kv_layer_geom") else None
        shapes = [(kvh, d) for kvh, d, _ in geom] if geom else None
        n_attn = len(shapes) if shapes else getattr(model, "num_kv_layers", model.cfg.num_layers)
        ring, R = None, 0
        if ring_chunk and geom:
            R = ring_pages_for(max(w for _, _, w in geom), ring_chunk)
            # a ring pays only where it is shorter than the longest context
            ring = [0 < w and R < cls.pages_for(max_len or (1 << 30)) for _, _, w in geom]
            if not any(ring):
                ring, R = None, 0
        if shapes:
            per_page = sum(2 * kvh * PAGE * d * es for (kvh, d), rg in zip(shapes, ring or [False] * len(shapes))
                           if not rg)
            ring_bytes = max_seqs * R * sum(2 * kvh * PAGE * d * es for (kvh, d), rg in zip(shapes, ring or [])
                                            if rg)
        else:
            per_page = 2 * max(n_attn, 1) * model.KVH * PAGE * model.D * es
            ring_bytes = 0
        if kv_bytes is not None:
            n = max(1, (kv_bytes - ring_bytes) // max(per_page, 1))
        else:
            n = cls.pages_for(max_tokens or 4096) + 1
        c = cls(max(n_attn, 1), n, model.KVH, model.D, dt, dev, kv_fp8, layer_shapes=shapes or None,
                layer_ring=ring, ring_pages=R, ring_seqs=max_seqs)
        n_lin = sum(1 for i in range(model.cfg.num_layers) if model.cfg.is_linear(i))
        if n_lin > 0:
            Hk, Dk, Hv, Dv = model.cfg.gdn_dims
            c.rec = RecurrentStatePool(n_lin, max_seqs, model.cfg.gdn_conv_dim, Hv, Dv, Dk,
                                       model.cfg.linear_conv_kernel_dim, dt, dev)
        return c


def ring_pages_for(window: int, chunk: int) -> int:
    """Ring pages that hold a `window`-token history plus a `chunk`-token
    step: the keys one step reads span at most window + chunk - 1 positions,
    i.e. ceil((window + chunk) / 16) + 1 pages, all distinct modulo R."""
    return -(-(window + chunk) // PAGE) + 2


class SequenceKV:
    """One request's KV pages. `num_tokens` = tokens whose K/V are written.
    With ring layers, `ring` holds the sequence's ring pages (at most
    ``cache.ring_pages``)."""

    def __init__(self, cache: PagedKVCache):
        self.cache = cache
        self.ring: list[int] = []
        self.pages: list[int] = []
        self.num_tokens = 0
        self.shared_prefix_pages = 0  # leading pages borrowed from the prefix cache
        self.state_slot = -1  # recurrent-state slot (hybrid models)

    def capacity(self) -> int:
        return len(self.pages) * PAGE

    def pages_needed(self, total_tokens: int) -> int:
        return max(0, PagedKVCache.pages_for(total_tokens) - len(self.pages))

    def ensure(self, total_tokens: int) -> bool:
        """Grow to hold `total_tokens`; False if the pool cannot supply pages."""
        rec = self.cache.rec
        new_slot = False
        if rec is not None and self.state_slot < 0:
            slot = rec.alloc()
            if slot is None:
                return False
            self.state_slot, new_slot = slot, True
        c = self.cache
        if c.ring_pages:
            rn = min(c.ring_pages, PagedKVCache.pages_for(total_tokens)) - len(self.ring)
            if rn > 0:
                if not c.ring_pool.can_alloc(rn):
                    return False
                self.ring.extend(c.ring_pool.alloc(rn))
        need = self.pages_needed(total_tokens)
        if need == 0:
            return True
        if not self.cache.pool.can_alloc(need):
            if new_slot:  # hold no state slot while waiting for pages
                rec.release(self.state_slot)
                self.state_slot = -1
            return False
        self.pages.extend(self.cache.pool.alloc(need))
        return True

    def ring_slot(self, pos: int) -> int:
        return self.ring[(pos // PAGE) % self.cache.ring_pages] * PAGE + pos % PAGE

    def ring_slots(self, start: int, n: int) -> list[int]:
        rg, R = self.ring, self.cache.ring_pages
        return [rg[(p // PAGE) % R] * PAGE + p % PAGE for p in range(start, start + n)]

    def ring_table(self, n: int):
        """Logical page table of the ring layers, `n` entries: page p -> ring[p % R]
        (entries past the written pages repeat ring pages; kernels never read them)."""
        import numpy as np

        rg = np.asarray(self.ring, dtype=np.int32)
        if rg.size == 0:
            return np.zeros(n, np.int32)
        idx = np.minimum(np.arange(n) % self.cache.ring_pages, rg.size - 1)
        return rg[idx]

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
        if self.ring:
            self.cache.ring_pool.decref(self.ring)
            self.ring = []
        self.pages = []
        self.num_tokens = 0
        self.shared_prefix_pages = 0
        if self.state_slot >= 0 and self.cache.rec is not None:
            self.cache.rec.release(self.state_slot)
        self.state_slot = -1
