"""RoPE variants as cos/sin tables.

Every rotary variant of the reference (MLXLMCommon/RoPEUtils.swift:86 default,
:164 Llama 3, :250 proportional, :367 YaRN, :402 dynamic NTK-alpha;
SuScaledRoPE.swift) changes only the per-dimension inverse frequencies and an
output scale, so each is reduced here to an ``inv_freq`` vector plus
``mscale``. The kernel side (qk_norm_rope_kv) reads one precomputed fp32 table
``[max_pos, rot_dim]`` (cos | sin), which makes every variant free at runtime.
"""
from __future__ import annotations

import math

import torch

from ..ops.reference import rope_cos_sin


def default_inv_freq(dim: int, base: float) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))


def llama3_inv_freq(dim, base, factor, low_freq_factor, high_freq_factor, original_max_pos):
    inv = default_inv_freq(dim, base)
    low_wl = original_max_pos / low_freq_factor
    high_wl = original_max_pos / high_freq_factor
    wl = 2 * math.pi / inv
    out = torch.where(wl > low_wl, inv / factor, inv)
    smooth = (original_max_pos / wl - low_freq_factor) / (high_freq_factor - low_freq_factor)
    mid = (1 - smooth) * out / factor + smooth * out
    is_mid = (wl >= high_wl) & (wl <= low_wl)
    return torch.where(is_mid, mid, out)


def yarn_inv_freq(dim, base, factor, original_max_pos, beta_fast=32.0, beta_slow=1.0, mscale=1.0,
                  mscale_all_dim=0.0, truncate=True):
    def corr_dim(n_rot):
        return (dim * math.log(original_max_pos / (n_rot * 2 * math.pi))) / (2 * math.log(base))

    low = corr_dim(beta_fast)
    high = corr_dim(beta_slow)
    if truncate:
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, dim - 1)
    if low == high:
        high += 0.001
    ramp = ((torch.arange(dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
    extrap = default_inv_freq(dim, base)
    interp = extrap / factor
    mask = 1 - ramp
    inv = interp * (1 - mask) + extrap * mask

    def get_mscale(scale, m):
        return 1.0 if scale <= 1 else 0.1 * m * math.log(scale) + 1.0

    ms = get_mscale(factor, mscale) / get_mscale(factor, mscale_all_dim) if mscale_all_dim else get_mscale(factor, mscale)
    return inv, ms


def dynamic_ntk_inv_freq(dim, base, alpha):
    return default_inv_freq(dim, base * alpha ** (dim / (dim - 2)))


def su_scaled_inv_freq(dim, base, short_factor):
    inv = default_inv_freq(dim, base)
    return inv / torch.tensor(short_factor, dtype=torch.float64)


def build_rope(head_dim: int, base: float, scaling: dict | None, max_pos: int, partial_rotary_factor: float = 1.0):
    """Returns (cos_sin table [max_pos, rot_dim] fp32, rot_dim)."""
    rot = int(head_dim * partial_rotary_factor)
    rot -= rot % 2
    mscale = 1.0
    kind = (scaling or {}).get("rope_type", (scaling or {}).get("type", "default")) if scaling else "default"
    if kind in ("default", None, "mrope"):  # mrope: the 1-D table of text positions (sections equal)
        inv = default_inv_freq(rot, base)
    elif kind == "linear":
        inv = default_inv_freq(rot, base) / float(scaling["factor"])
    elif kind == "llama3":
        inv = llama3_inv_freq(rot, base, float(scaling["factor"]), float(scaling.get("low_freq_factor", 1.0)),
                              float(scaling.get("high_freq_factor", 4.0)),
                              int(scaling.get("original_max_position_embeddings", 8192)))
    elif kind == "yarn":
        inv, mscale = yarn_inv_freq(rot, base, float(scaling["factor"]),
                                    int(scaling.get("original_max_position_embeddings", 4096)),
                                    float(scaling.get("beta_fast", 32.0)), float(scaling.get("beta_slow", 1.0)),
                                    float(scaling.get("mscale", 1.0)), float(scaling.get("mscale_all_dim", 0.0)),
                                    bool(scaling.get("truncate", True)))
    elif kind == "dynamic":
        alpha = float(scaling.get("alpha", scaling.get("factor", 1.0)))
        inv = dynamic_ntk_inv_freq(rot, base, alpha)
    elif kind in ("su", "longrope"):
        inv = su_scaled_inv_freq(rot, base, scaling["short_factor"])
        f = float(scaling.get("factor", 1.0))
        omp = int(scaling.get("original_max_position_embeddings", max_pos))
        if f > 1:
            mscale = math.sqrt(1 + math.log(f) / math.log(omp))
    elif kind == "proportional":
        inv = default_inv_freq(rot, base) * float(scaling.get("factor", 1.0))
    else:
        raise ValueError(f"unsupported rope scaling {kind}")
    return rope_cos_sin(inv, max_pos, mscale), rot
