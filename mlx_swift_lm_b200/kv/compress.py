"""KV-cache compression schemes for the legacy single-sequence path.

Parity: the ``kvScheme`` strings of MLXLMCommon/Evaluate.swift:168-194 -
``affine4`` / ``affine8``; TurboQuant ``turbo<K>v<V>`` (keys x values:
K = 0 keeps keys in full precision, 8 is 8-bit affine, 2-4 is the rotated
codebook quantiser; ``turbo4`` / ``turbo3`` / ``turbo2`` use it for both);
variance-normalised ``varn<K>v<V>`` with 128-token tiles (``t32`` / ``t64``
suffixes pick the tile), ``varn`` = ``varn4v2``.

Both quantisers are written here from their published methods:

* TurboQuant (Zandieh et al., 2025): a vector is split into its norm and
  direction; the direction is rotated by a fixed random orthogonal transform
  (random signs followed by a normalised Walsh-Hadamard transform), after
  which each coordinate is close to N(0, 1/d) and is quantised independently
  with the Lloyd-Max codebook of that distribution (computed below by Lloyd
  iterations on a fine grid).
* Variance-normalised tiles (KVarN): within a tile of tokens each channel is
  centred and scaled by its own mean and standard deviation, and the
  normalised tile is quantised with uniform per-token codes; the per-channel
  statistics are stored per tile. Tokens of an unfinished tile stay in full
  precision until the tile fills.
"""
from __future__ import annotations

import functools
import math
import re

import torch

from ..ops import quant


# ---------------------------------------------------------------------- TurboQuant
@functools.lru_cache(maxsize=None)
def lloyd_max_gaussian(bits: int, iters: int = 200) -> torch.Tensor:
    """Lloyd-Max reconstruction levels of N(0, 1) for 2**bits levels."""
    n = 1 << bits
    x = torch.linspace(-6, 6, 24001, dtype=torch.float64)
    pdf = torch.exp(-0.5 * x * x)
    levels = torch.linspace(-2.0, 2.0, n, dtype=torch.float64) * (1.0 if bits > 1 else 0.8)
    for _ in range(iters):
        edges = (levels[1:] + levels[:-1]) / 2
        idx = torch.bucketize(x, edges)
        num = torch.zeros(n, dtype=torch.float64).index_add_(0, idx, pdf * x)
        den = torch.zeros(n, dtype=torch.float64).index_add_(0, idx, pdf)
        levels = torch.where(den > 0, num / den.clamp(min=1e-300), levels)
    return levels.float()


def _hadamard(x: torch.Tensor) -> torch.Tensor:
    """Normalised Walsh-Hadamard transform along the last dim (a power of 2)."""
    d = x.shape[-1]
    h = 1
    y = x.clone()
    while h < d:
        y = y.reshape(*y.shape[:-1], d // (2 * h), 2, h)
        a, b = y[..., 0, :], y[..., 1, :]
        y = torch.stack([a + b, a - b], -2).reshape(*x.shape)
        h *= 2
    return y / math.sqrt(d)


@functools.lru_cache(maxsize=None)
def _signs(d: int, seed: int = 0x7B5) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + d)
    return (torch.randint(0, 2, (d,), generator=g) * 2 - 1).float()


def turbo_quantize(x: torch.Tensor, bits: int):
    """x [..., d] -> (codes uint8 [..., d], norms fp32 [...])."""
    d = x.shape[-1]
    xf = x.float()
    norm = xf.norm(dim=-1)
    u = xf / norm.clamp(min=1e-12)[..., None]
    r = _hadamard(u * _signs(d).to(x.device)) * math.sqrt(d)  # coordinates ~ N(0, 1)
    lv = lloyd_max_gaussian(bits).to(x.device)
    codes = torch.bucketize(r, (lv[1:] + lv[:-1]) / 2).to(torch.uint8)
    return codes, norm


def turbo_dequantize(codes: torch.Tensor, norm: torch.Tensor, bits: int, dtype=torch.float32) -> torch.Tensor:
    d = codes.shape[-1]
    lv = lloyd_max_gaussian(bits).to(codes.device)
    r = lv[codes.long()] / math.sqrt(d)
    u = _hadamard(r) * _signs(d).to(codes.device)  # the transform is its own inverse up to the signs
    return (u * norm[..., None]).to(dtype)


# ---------------------------------------------------------------------- variance-normalised tiles
def varn_quantize(x: torch.Tensor, bits: int):
    """A tile x [T, H, D] -> (codes uint8 [T, H, D], per-token scale / offset
    [T, H], per-channel mean / std [H, D])."""
    xf = x.float()
    mu = xf.mean(0)
    sd = xf.std(0, unbiased=False).clamp(min=1e-6)
    z = (xf - mu) / sd
    lo, hi = z.amin(-1), z.amax(-1)
    levels = (1 << bits) - 1
    scale = ((hi - lo) / levels).clamp(min=1e-8)
    q = torch.round((z - lo[..., None]) / scale[..., None]).clamp(0, levels).to(torch.uint8)
    return q, scale, lo, mu, sd


def varn_dequantize(q, scale, lo, mu, sd, dtype=torch.float32):
    z = q.float() * scale[..., None] + lo[..., None]
    return (z * sd + mu).to(dtype)


# ---------------------------------------------------------------------- schemes
_TURBO = re.compile(r"^turbo(\d)(?:v(\d))?$")
_VARN = re.compile(r"^varn(?:(\d)(?:v(\d))?)?(?:t(32|64|128))?$")


def parse_scheme(s: str) -> dict:
    """{kind, k_bits, v_bits, tile}; raises on an unknown scheme."""
    if s in ("affine4", "affine8"):
        b = int(s[-1])
        return {"kind": "affine", "k_bits": b, "v_bits": b, "tile": 0}
    m = _TURBO.match(s)
    if m:
        kb = int(m.group(1))
        vb = int(m.group(2)) if m.group(2) else kb
        if kb not in (0, 2, 3, 4, 8) or vb not in (2, 3, 4):
            raise ValueError(f"unsupported TurboQuant scheme {s!r}")
        return {"kind": "turbo", "k_bits": kb, "v_bits": vb, "tile": 0}
    m = _VARN.match(s)
    if m:
        kb = int(m.group(1)) if m.group(1) else 4
        vb = int(m.group(2)) if m.group(2) else (2 if not m.group(1) else kb)
        if kb not in (2, 4) or vb not in (2, 4):
            raise ValueError(f"unsupported variance-normalised scheme {s!r}")
        return {"kind": "varn", "k_bits": kb, "v_bits": vb, "tile": int(m.group(3) or 128)}
    raise ValueError(f"unknown KV scheme {s!r}")


class _Codec:
    """Encode / decode one tensor kind (keys or values) of a scheme."""

    def __init__(self, kind: str, bits: int):
        self.kind, self.bits = kind, bits

    def encode(self, x):
        if self.kind == "full" or self.bits == 0:
            return ("full", x.clone())
        if self.kind == "affine" or (self.kind == "turbo" and self.bits == 8):
            n, h, d = x.shape
            gs = min(64, d)
            p, s, b = quant.affine_quantize(x.reshape(n * h, d).float(), gs, self.bits)
            return ("affine", p, s, b, x.shape, gs)
        if self.kind == "turbo":
            c, nrm = turbo_quantize(x, self.bits)
            return ("turbo", c, nrm)
        return ("varn",) + varn_quantize(x, self.bits)

    def decode(self, e, dtype):
        if e[0] == "full":
            return e[1].to(dtype)
        if e[0] == "affine":
            _, p, s, b, shape, gs = e
            return quant.dequantize(p, s, b, "affine", gs, self.bits, torch.float32).reshape(shape).to(dtype)
        if e[0] == "turbo":
            return turbo_dequantize(e[1], e[2], self.bits, dtype)
        return varn_dequantize(*e[1:], dtype=dtype)

    @staticmethod
    def nbytes(e) -> int:
        return sum(t.numel() * t.element_size() for t in e[1:] if isinstance(t, torch.Tensor))


class CompressedKVCache:
    """Legacy cache storing K/V under a compression scheme; ``update``
    returns the decoded keys / values the attention reads."""

    def __init__(self, num_layers: int, scheme: str):
        self.scheme = scheme
        p = parse_scheme(scheme)
        kind = p["kind"]
        self.tile = p["tile"]
        self.kc = _Codec("full" if (kind == "turbo" and p["k_bits"] == 0) else kind, p["k_bits"])
        self.vc = _Codec(kind, p["v_bits"])
        self.blocks = [[] for _ in range(num_layers)]  # encoded (K, V, n_tokens)
        self.tail = [None] * num_layers  # varn: tokens of the unfinished tile (full precision)
        self.offset = 0
        self.k = [None] * num_layers  # interface compatibility (unused)

    def update(self, layer, k, v):
        if self.tile:
            tk, tv = self.tail[layer] if self.tail[layer] is not None else (k[:0], v[:0])
            tk, tv = torch.cat([tk, k]), torch.cat([tv, v])
            while tk.shape[0] >= self.tile:
                self.blocks[layer].append((self.kc.encode(tk[:self.tile]), self.vc.encode(tv[:self.tile]),
                                           self.tile))
                tk, tv = tk[self.tile:], tv[self.tile:]
            self.tail[layer] = (tk, tv)
        else:
            self.blocks[layer].append((self.kc.encode(k), self.vc.encode(v), k.shape[0]))
        ks = [self.kc.decode(b[0], k.dtype) for b in self.blocks[layer]]
        vs = [self.vc.decode(b[1], v.dtype) for b in self.blocks[layer]]
        if self.tile and self.tail[layer] is not None:
            ks.append(self.tail[layer][0])
            vs.append(self.tail[layer][1])
        return torch.cat(ks), torch.cat(vs)

    def nbytes(self) -> int:
        n = 0
        for li, bl in enumerate(self.blocks):
            for ek, ev, _ in bl:
                n += _Codec.nbytes(ek) + _Codec.nbytes(ev)
            if self.tail[li] is not None:
                n += sum(t.numel() * t.element_size() for t in self.tail[li])
        return n

    def trim(self, n: int):
        raise NotImplementedError("compressed caches do not rewind (re-prefill instead)")
