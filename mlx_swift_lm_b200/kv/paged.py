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
                 dtype=torch.bfloat16, device="cpu", kv_fp8: bool = False, layer_shapes=None):
        """`layer_shapes`: optional (KVH, D) of every KV layer; layers of one
        shape share a slab. Default: every layer (num_kv_heads, head_dim)."""
        shapes = [tuple(x) for x in layer_shapes] if layer_shapes else [(num_kv_heads, head_dim)] * num_layers
        self.num_layers = len(shapes)
        self.num_pages = num_pages
        self.device = torch.device(device)
        self.kv_fp8 = kv_fp8
        sdt = torch.float8_e4m3fn if kv_fp8 else dtype
        # group g: layers of shape group_shapes[g]; _where[li] = (g, index within the group)
        self.group_shapes: list[tuple[int, int]] = []
        self._where: list[tuple[int, int]] = []
        counts: dict[tuple[int, int], int] = {}
        for sh in shapes:
            if sh not in counts:
                counts[sh] = 0
                self.group_shapes.append(sh)
            self._where.append((self.group_shapes.index(sh), counts[sh]))
            counts[sh] += 1
        self.gk, self.gv = [], []
        for sh in self.group_shapes:
            kvh, d = sh
            shape = (counts[sh], num_pages, kvh, PAGE, d)
            self.gk.append(torch.zeros(shape, dtype=sdt, device=self.device))
            self.gv.append(torch.zeros(shape, dtype=sdt, device=self.device))
        # the first group's slabs and geometry (single-group models: the whole cache)
        self.k, self.v = self.gk[0], self.gv[0]
        self.kvh, self.head_dim = self.group_shapes[0]
        self.layer_shapes = shapes
        kvh_max = max(k for k, _ in shapes)
        if kv_fp8:
            # per-layer, per-KV-head dequantisation scales (stored = x / scale)
            self.k_scales = torch.ones((self.num_layers, kvh_max), dtype=torch.float32, device=self.device)
            self.v_scales = torch.ones((self.num_layers, kvh_max), dtype=torch.float32, device=self.device)
        else:
            self.k_scales = self.v_scales = None
        self.pool = _b200host.PagePool(num_pages)
        es = self.k.element_size()
        self.page_bytes = sum(2 * kvh * PAGE * d * es for kvh, d in shapes)
        self.rec: RecurrentStatePool | None = None

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
                  device=None, max_seqs: int = 64):
        """Size the pool by a token budget or a byte budget. Only attention
        layers hold pages; linear-attention layers get `max_seqs` state slots."""
        dev = device or model.device
        dt = model.dtype
        es = 1 if kv_fp8 else torch.empty((), dtype=dt).element_size()
        geom = model.kv_layer_geom() if hasattr(model, "kv_layer_geom") else None
        shapes = [(kvh, d) for kvh, d, _ in geom] if geom else None
        n_attn = len(shapes) if shapes else getattr(model, "num_kv_layers", model.cfg.num_layers)
        if shapes:
            per_page = sum(2 * kvh * PAGE * d * es for kvh, d in shapes)
        else:
            per_page = 2 * max(n_attn, 1) * model.KVH * PAGE * model.D * es
        if kv_bytes is not None:
            n = max(1, kv_bytes // per_page)
        else:
            n = cls.pages_for(max_tokens or 4096) + 1
        c = cls(max(n_attn, 1), n, model.KVH, model.D, dt, dev, kv_fp8, layer_shapes=shapes or None)
        n_lin = sum(1 for i in range(model.cfg.num_layers) if model.cfg.is_linear(i))
        if n_lin > 0:
            Hk, Dk, Hv, Dv = model.cfg.gdn_dims
            c.rec = RecurrentStatePool(n_lin, max_seqs, model.cfg.gdn_conv_dim, Hv, Dv, Dk,
                                       model.cfg.linear_conv_kernel_dim, dt, dev)
        return c


class SequenceKV:
    """One request's KV pages. `num_tokens` = tokens whose K/V are written."""

    def __init__(self, cache: PagedKVCache):
        self.cache = cache
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
        if self.state_slot >= 0 and self.cache.rec is not None:
            self.cache.rec.release(self.state_slot)
        self.state_slot = -1
