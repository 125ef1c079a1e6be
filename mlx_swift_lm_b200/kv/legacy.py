"""Legacy single-sequence KV caches and prompt-cache files.

Parity: MLXLMCommon/KVCache.swift - ``KVCacheSimple`` (:470, grows by
concatenation; :class:`..models.decoder.DenseKVCache`), ``RotatingKVCache``
(:641, a sliding window that keeps the first tokens), ``QuantizedKVCache``
(:1179, affine codes per group along the head dimension), ``ChunkedKVCache``
(:1486, attention within fixed chunks), ``CacheList`` (:1993) and
``savePromptCache`` / ``loadPromptCache`` (:2248) to safetensors.

Every cache implements ``update(layer, k, v) -> (keys, values)`` (the keys a
new chunk attends to, k/v [n, KVH, D]), ``key_positions(layer)`` (absolute
positions of those keys, for the causal mask), ``offset`` and ``trim(n)``;
:func:`save_prompt_cache` / :func:`load_prompt_cache` write and read them.
They serve the dense single-request path (``DecoderLM.forward_dense``,
``api.generate.TokenIterator``).
"""
from __future__ import annotations

import json

import torch

from ..models.decoder import DenseKVCache
from ..ops import quant


class _PositionedCache(DenseKVCache):
    """Dense cache that also records each stored key's absolute position."""

    def __init__(self, num_layers: int):
        super().__init__(num_layers)
        self.pos = [None] * num_layers

    def _append(self, layer, k, v):
        n = k.shape[0]
        p0 = self.offset
        new_pos = torch.arange(p0, p0 + n, device=k.device)
        if self.k[layer] is None:
            self.k[layer], self.v[layer], self.pos[layer] = k, v, new_pos
        else:
            self.k[layer] = torch.cat([self.k[layer], k], 0)
            self.v[layer] = torch.cat([self.v[layer], v], 0)
            self.pos[layer] = torch.cat([self.pos[layer], new_pos], 0)

    def key_positions(self, layer: int):
        return self._last_pos[layer] if hasattr(self, "_last_pos") else self.pos[layer]

    def trim(self, n: int):
        n = min(n, self.offset)
        for i in range(len(self.k)):
            if self.k[i] is not None:
                keep = self.pos[i] < self.offset - n
                self.k[i], self.v[i], self.pos[i] = self.k[i][keep], self.v[i][keep], self.pos[i][keep]
        self.offset -= n
        return n


class RotatingKVCache(_PositionedCache):
    """Keeps the first `keep` tokens and the most recent `max_size - keep`.
    A multi-token update attends to everything kept so far plus the whole
    new chunk (each query masked causally by position), then the store is cut
    back to the window."""

    def __init__(self, num_layers: int, max_size: int, keep: int = 4):
        super().__init__(num_layers)
        self.max_size, self.keep = max_size, keep
        self._last_pos = [None] * num_layers

    def update(self, layer, k, v):
        self._append(layer, k, v)
        K, V, P = self.k[layer], self.v[layer], self.pos[layer]
        self._last_pos[layer] = P
        if K.shape[0] > self.max_size:
            sel = torch.cat([torch.arange(self.keep, device=K.device),
                             torch.arange(K.shape[0] - (self.max_size - self.keep), K.shape[0], device=K.device)])
            self.k[layer], self.v[layer], self.pos[layer] = K[sel], V[sel], P[sel]
        return K, V


class ChunkedKVCache(_PositionedCache):
    """Attention within fixed chunks of `chunk_size` positions: a query sees
    only keys of its own chunk; the store keeps the current chunk."""

    def __init__(self, num_layers: int, chunk_size: int):
        super().__init__(num_layers)
        self.chunk_size = chunk_size
        self._last_pos = [None] * num_layers

    def update(self, layer, k, v):
        self._append(layer, k, v)
        K, V, P = self.k[layer], self.v[layer], self.pos[layer]
        self._last_pos[layer] = P
        start = ((self.offset + k.shape[0] - 1) // self.chunk_size) * self.chunk_size
        keep = P >= start
        self.k[layer], self.v[layer], self.pos[layer] = K[keep], V[keep], P[keep]
        return K, V

    def chunk_mask(self, q_pos: torch.Tensor, k_pos: torch.Tensor) -> torch.Tensor:
        return (k_pos[None, :] // self.chunk_size) == (q_pos[:, None] // self.chunk_size)


class QuantizedKVCache(_PositionedCache):
    """K/V stored only as affine `bits`-bit codes with a scale and bias per
    `group_size` head-dim values (MLX quantize layout); each update returns
    the dequantised keys / values a quantised attention would read."""

    def __init__(self, num_layers: int, bits: int = 8, group_size: int = 64):
        super().__init__(num_layers)
        self.bits, self.gs = bits, group_size
        self.codes = [None] * num_layers  # per layer: [K, V] x (packed [n, h, w], scales, biases)

    def _quant(self, x):
        n, h, d = x.shape
        gs = min(self.gs, d)
        packed, sc, bi = quant.affine_quantize(x.reshape(n * h, d).float(), gs, self.bits)
        return packed.reshape(n, h, -1), sc.reshape(n, h, -1), bi.reshape(n, h, -1)

    def _deq(self, c, d, dtype):
        packed, sc, bi = c
        n, h = packed.shape[:2]
        gs = min(self.gs, d)
        w = quant.dequantize(packed.reshape(n * h, -1), sc.reshape(n * h, -1), bi.reshape(n * h, -1), "affine", gs,
                             self.bits, torch.float32)
        return w.reshape(n, h, d).to(dtype)

    def update(self, layer, k, v):
        n = k.shape[0]
        new = [self._quant(k), self._quant(v)]
        pos = torch.arange(self.offset, self.offset + n, device=k.device)
        if self.codes[layer] is None:
            self.codes[layer], self.pos[layer] = new, pos
        else:
            self.codes[layer] = [tuple(torch.cat([a, b], 0) for a, b in zip(old, nw))
                                 for old, nw in zip(self.codes[layer], new)]
            self.pos[layer] = torch.cat([self.pos[layer], pos], 0)
        d = k.shape[-1]
        return self._deq(self.codes[layer][0], d, k.dtype), self._deq(self.codes[layer][1], d, v.dtype)

    def trim(self, n: int):
        n = min(n, self.offset)
        for i, c in enumerate(self.codes):
            if c is not None:
                keep = self.pos[i] < self.offset - n
                self.codes[i] = [tuple(t[keep] for t in kv) for kv in c]
                self.pos[i] = self.pos[i][keep]
        self.offset -= n
        return n

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for c in self.codes if c is not None for kv in c for t in kv)


class CacheList:
    """One cache object per layer (mixed cache kinds in one model)."""

    def __init__(self, caches: list):
        self.caches = list(caches)
        self.offset = 0

    def update(self, layer, k, v):
        c = self.caches[layer]
        c.offset = self.offset
        return c.update(0 if isinstance(c, DenseKVCache) and len(c.k) == 1 else layer, k, v)

    def key_positions(self, layer):
        c = self.caches[layer]
        return c.key_positions(0 if len(c.k) == 1 else layer) if hasattr(c, "key_positions") else None

    def trim(self, n):
        for c in self.caches:
            c.offset = self.offset
            c.trim(n)
        self.offset -= min(n, self.offset)
        return n


# ---------------------------------------------------------------------- prompt cache files
def save_prompt_cache(path: str, cache, metadata: dict | None = None):
    """Write a dense / rotating / chunked cache (keys, values, positions,
    offset and kind) to a safetensors file with string metadata."""
    from ..loader.safetensors import save_safetensors

    t = {}
    if isinstance(cache, QuantizedKVCache):
        for i, c in enumerate(cache.codes):
            if c is not None:
                for name, kv in zip(("keys", "values"), c):
                    for part, x in zip(("codes", "scales", "biases"), kv):
                        t[f"layers.{i}.{name}.{part}"] = x
                t[f"layers.{i}.positions"] = cache.pos[i]
    for i in range(len(cache.k)):
        if cache.k[i] is not None:
            t[f"layers.{i}.keys"] = cache.k[i]
            t[f"layers.{i}.values"] = cache.v[i]
            if getattr(cache, "pos", None) is not None and cache.pos[i] is not None:
                t[f"layers.{i}.positions"] = cache.pos[i]
    info = {"kind": type(cache).__name__, "offset": cache.offset, "num_layers": len(cache.k)}
    for a in ("max_size", "keep", "chunk_size", "bits", "gs"):
        if hasattr(cache, a):
            info[a] = getattr(cache, a)
    md = {"cache": json.dumps(info)}
    for k, v in (metadata or {}).items():
        md[k] = v
    save_safetensors(path, t, md)


def load_prompt_cache(path: str, device="cpu"):
    """(cache, user metadata) from :func:`save_prompt_cache`."""
    from ..loader.safetensors import load_safetensors

    t, md = load_safetensors(path)
    info = json.loads(md.pop("cache"))
    n = info["num_layers"]
    kind = info["kind"]
    if kind == "RotatingKVCache":
        c = RotatingKVCache(n, info["max_size"], info["keep"])
    elif kind == "ChunkedKVCache":
        c = ChunkedKVCache(n, info["chunk_size"])
    elif kind == "QuantizedKVCache":
        c = QuantizedKVCache(n, info["bits"], info["gs"])
    elif kind == "DenseKVCache":
        c = DenseKVCache(n)
    else:
        c = _PositionedCache(n)
    for i in range(n):
        if isinstance(c, QuantizedKVCache) and f"layers.{i}.keys.codes" in t:
            c.codes[i] = [tuple(t[f"layers.{i}.{nm}.{part}"].to(device) for part in ("codes", "scales", "biases"))
                          for nm in ("keys", "values")]
            c.pos[i] = t[f"layers.{i}.positions"].to(device)
        if f"layers.{i}.keys" in t:
            c.k[i] = t[f"layers.{i}.keys"].to(device)
            c.v[i] = t[f"layers.{i}.values"].to(device)
            if hasattr(c, "pos"):
                c.pos[i] = t[f"layers.{i}.positions"].to(device)
    c.offset = info["offset"]
    return c, md
