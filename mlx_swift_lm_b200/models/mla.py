"""Multi-head latent attention (DeepSeek V2 / V3, GLM-4.7-Flash) on the paged cache.

Per layer (MLXLLM/Models/DeepseekV3.swift, GLM4MOELite.swift):

    q      = q_b(rmsnorm(q_a(x)))          (or q_proj(x) without a query LoRA)
             -> per head [q_nope (qk_nope) | q_pe (qk_rope)]
    c, kpe = kv_a(x) = [latent (kv_lora) | k_pe (qk_rope, shared by all heads)]
    k_nope, v = kv_b(rmsnorm(c))           per head [qk_nope | v_head]
    k      = [k_nope | rope(k_pe)],  q = [q_nope | rope(q_pe)]   (interleaved rotary)
    out    = o_proj(softmax(q k^T * scale) v)

The cache holds the decompressed per-head K and V, both padded with zeros to
one head dim that the paged kernels serve (``cfg.head_dim``, 256 for the
192 / 128 split of DeepSeek V3): zero channels leave q.k unchanged and the
padded output channels are dropped before o_proj. This trades cache bytes
for reuse of the paged decode / prefill kernels; the absorbed form (attention
in the latent space) is not built.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..ops import reference as ref


def mla_dims(cfg):
    e = cfg.extra
    return e["mla_q_lora"], e["mla_kv_lora"], e["mla_qk_nope"], e["mla_qk_rope"], e["mla_v"]


def config_from_hf(cfg, hf: dict):
    """MLA switches of a DeepSeek-style config.json."""
    nope, rope_d, vd = hf["qk_nope_head_dim"], hf["qk_rope_head_dim"], hf["v_head_dim"]
    need = max(nope + rope_d, vd)
    dp = next((d for d in (64, 128, 256) if d >= need), None)
    if dp is None:
        raise NotImplementedError(f"MLA head dims {nope}+{rope_d}/{vd} exceed the paged kernels' 256")
    cfg.extra.update(mla=True, mla_q_lora=hf.get("q_lora_rank") or 0, mla_kv_lora=hf["kv_lora_rank"],
                     mla_qk_nope=nope, mla_qk_rope=rope_d, mla_v=vd)
    cfg.head_dim = dp
    cfg.num_kv_heads = cfg.num_heads
    cfg.partial_rotary_factor = rope_d / dp  # the rotary table covers the q_pe / k_pe channels
    cfg.rope_interleaved = True
    scale = (nope + rope_d) ** -0.5
    rs = cfg.rope_scaling or {}
    if rs.get("rope_type", rs.get("type")) == "yarn" and rs.get("mscale_all_dim"):
        f = float(rs["factor"])
        m = 0.1 * float(rs["mscale_all_dim"]) * math.log(f) + 1.0 if f > 1 else 1.0
        scale *= m * m
    cfg.attn_scale = scale


def init_random(model, L, rn, ones):
    cfg = model.cfg
    ql, kl, nope, rope_d, vd = mla_dims(cfg)
    H, hd = cfg.num_heads, cfg.hidden_size
    if ql:
        L.mla_q_a, L.mla_q_a_norm, L.mla_q_b = rn(ql, hd), ones(ql), rn(H * (nope + rope_d), ql)
    else:
        L.mla_q_b = rn(H * (nope + rope_d), hd)
    L.mla_kv_a, L.mla_kv_a_norm, L.mla_kv_b = rn(kl + rope_d, hd), ones(kl), rn(H * (nope + vd), kl)
    L.wo = rn(hd, H * vd)


def qkv(model, L, h, positions):
    """(q, k, v) [T, H, Dp] of the tokens in h, rotated at `positions`, padded to Dp."""
    cfg = model.cfg
    ql, kl, nope, rope_d, vd = mla_dims(cfg)
    H, Dp, eps = model.H, model.D, cfg.rms_norm_eps
    T = h.shape[0]
    if L.mla_q_a is not None:
        q = ops.gemm(ops.rmsnorm(ops.gemm(h, L.mla_q_a), L.mla_q_a_norm, eps), L.mla_q_b)
    else:
        q = ops.gemm(h, L.mla_q_b)
    q = q.view(T, H, nope + rope_d)
    kva = ops.gemm(h, L.mla_kv_a)
    c = ops.rmsnorm(kva[:, :kl].contiguous(), L.mla_kv_a_norm, eps)
    kv = ops.gemm(c, L.mla_kv_b).view(T, H, nope + vd)
    dt = q.dtype
    qpe = ref.apply_rope_ref(q[..., nope:].float(), positions, model.cos_sin, rope_d, True).to(dt)
    kpe = ref.apply_rope_ref(kva[:, None, kl:].float(), positions, model.cos_sin, rope_d, True).to(dt)
    qf = torch.zeros(T, H, Dp, dtype=dt, device=h.device)
    kf, vf = torch.zeros_like(qf), torch.zeros_like(qf)
    qf[..., :nope] = q[..., :nope]
    qf[..., nope:nope + rope_d] = qpe
    kf[..., :nope] = kv[..., :nope]
    kf[..., nope:nope + rope_d] = kpe.expand(T, H, rope_d)
    vf[..., :vd] = kv[..., nope:]
    return qf, kf, vf


def attention(model, L, h, fb, kv_cache, li: int, attn):
    """Paged MLA of one layer; returns o_proj of the attention output."""
    cfg = model.cfg
    ql, kl, nope, rope_d, vd = mla_dims(cfg)
    T, nd = fb.num_tokens, fb.num_decode
    H, Dp = model.H, model.D
    ki = model.kv_index[li] if model.kv_index else li
    q, k, v = qkv(model, L, h, fb.positions)
    kc, vc = kv_cache.layer(ki)
    # append K/V at the tokens' slots (no further norm / rotary: rot_dim 0)
    packed = torch.cat([q.reshape(T, H * Dp), k.reshape(T, H * Dp), v.reshape(T, H * Dp)], 1)
    slots, dec_pt, pf_pt = fb.tables(kv_cache, ki)
    q = ops.qk_norm_rope_kv(packed, fb.positions, slots, model.cos_sin, 0, False, None, None, cfg.rms_norm_eps,
                            kc, vc, H, H, Dp, kv_cache.k_scale(ki), kv_cache.v_scale(ki))
    win = cfg.window(li)
    if nd:
        ops.paged_decode(q[:nd], kc, vc, dec_pt, fb.dec_seq_lens, cfg.scale, win, None, 0.0,
                         kv_cache.k_scale(ki), kv_cache.v_scale(ki), fb.dec_max_parts, out=attn[:nd])
    if T > nd:
        ops.paged_prefill(q[nd:], kc, vc, pf_pt, fb.pf_cu_q, fb.pf_pos0, cfg.scale, win, None, 0.0,
                          kv_cache.k_scale(ki), kv_cache.v_scale(ki), fb.pf_cu_q_host, out=attn[nd:])
    a2 = attn.view(T, H, Dp)[..., :vd].reshape(T, H * vd).contiguous()
    return model._attn_out(L, a2)


def dense_attention(model, L, h, cache, li: int, positions):
    """Single-sequence MLA with the dense concatenating cache (legacy path)."""
    cfg = model.cfg
    ql, kl, nope, rope_d, vd = mla_dims(cfg)
    T = h.shape[0]
    q, k, v = qkv(model, L, h, positions)
    ki = model.kv_index[li] if model.kv_index else li
    kk, vv = cache.update(ki, k, v)
    a = ref.attention_rows_ref(q.float(), kk.float(), vv.float(), positions, kk.shape[0], cfg.scale,
                               cfg.window(li), None, 0.0).to(h.dtype)
    a2 = a[..., :vd].reshape(T, model.H * vd).contiguous()
    return model._attn_out(L, a2)
