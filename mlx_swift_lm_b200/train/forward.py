"""Differentiable forward of a dense :class:`DecoderLM` with unfused LoRA /
DoRA adapters, for adapter training.

Serving runs the fused sm_100a kernels, which have no backward. Training of
adapters needs gradients only for the small adapter matrices, so it runs this
plain-PyTorch forward (autograd; cuBLAS on CUDA, any device works) over the
model's frozen weights in their fused layouts: the LoRA terms are added into
the fused q|k|v and interleaved gate/up outputs at the matching columns.
Parity: LoRALinear.callAsFunction (LoRA+Layers.swift:109: y + s * (dropout(x) A) B)
and DoRA's forward (DoRA+Layers.swift:13, norm of the adapted weight held
constant for the gradient).
Dense decoders with tensor-parallel world 1 only.
"""
from __future__ import annotations

import torch
import torch.nn.functional as Fn

from ..adapters.lora import LoRAContainer
from ..ops.reference import apply_rope_ref, attention_rows_ref


def _gate_up_index(F: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    j = torch.arange(F, device=device)
    g = (j // 64) * 128 + j % 64
    return g, g + 64


def _rms(x, w, eps, offset_one=False):
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    ww = w.float() + (1.0 if offset_one else 0.0)
    return xf * inv * ww


class TrainableLoRA:
    """Adapter matrices of a :class:`LoRAContainer` as trainable leaves."""

    def __init__(self, adapter: LoRAContainer, device, train_magnitude: bool = True):
        self.adapter = adapter
        self.scale = adapter.configuration.lora_parameters.scale
        self.dropout = adapter.configuration.lora_parameters.dropout
        self.dora = adapter.configuration.fine_tune_type == "dora"
        self.params: dict = {}
        for key, ent in adapter.tensors.items():
            a = ent["a"].to(device).float().requires_grad_(True)
            b = ent["b"].to(device).float().requires_grad_(True)
            m = None
            if ent.get("m") is not None:
                m = ent["m"].to(device).float().requires_grad_(train_magnitude)
            self.params[key] = {"a": a, "b": b, "m": m}

    def parameters(self):
        for ent in self.params.values():
            yield ent["a"]
            yield ent["b"]
            if ent["m"] is not None and ent["m"].requires_grad:
                yield ent["m"]

    def write_back(self):
        """Copy the trained values into the container (CPU fp32)."""
        for key, ent in self.params.items():
            dst = self.adapter.tensors[key]
            dst["a"] = ent["a"].detach().float().cpu()
            dst["b"] = ent["b"].detach().float().cpu()
            if ent["m"] is not None:
                dst["m"] = ent["m"].detach().float().cpu()

    def delta(self, x, key, w_rows, training: bool):
        """(s * dropout(x) A^T B^T, DoRA column scale or None) for one projection."""
        ent = self.params[key]
        xd = Fn.dropout(x, self.dropout, training) if self.dropout > 0 else x
        z = (xd @ ent["a"].t()) @ ent["b"].t() * self.scale
        if not self.dora:
            return z, None
        with torch.no_grad():
            v = w_rows.float() + self.scale * (ent["b"] @ ent["a"])
            nrm = v.pow(2).sum(1).sqrt().clamp_min(1e-12)
        return z, ent["m"] / nrm


def _proj_qkv(model, L, li, x, lora, training):
    y = x @ L.wqkv.float().t()
    if L.bqkv is not None:
        y = y + L.bqkv.float()
    if lora is None:
        return y
    qn, kn = model.H * model.D, model.KVH * model.D
    parts = (("self_attn.q_proj", 0, qn), ("self_attn.k_proj", qn, qn + kn), ("self_attn.v_proj", qn + kn, qn + 2 * kn))
    cols = []
    for key, lo, hi in parts:
        seg = y[:, lo:hi]
        if (li, key) in lora.params:
            z, sc = lora.delta(x, (li, key), L.wqkv[lo:hi], training)
            seg = seg + z
            if sc is not None:
                b = L.bqkv[lo:hi].float() if L.bqkv is not None else 0.0
                seg = (seg - b) * sc + b
        cols.append(seg)
    return torch.cat(cols, dim=1)


def _proj_plain(L_w, L_b, x, lora, key, training):
    y = x @ L_w.float().t()
    if lora is not None and key in lora.params:
        z, sc = lora.delta(x, key, L_w, training)
        y = y + z
        if sc is not None:
            y = y * sc
    if L_b is not None:
        y = y + L_b.float()
    return y


def _mlp(model, L, li, x, lora, training):
    cfg = model.cfg
    y = x @ L.wgu.float().t()
    F = L.wgu.shape[0] // 2
    gi, ui = _gate_up_index(F, x.device)
    g, u = y[:, gi], y[:, ui]
    if lora is not None:
        for key, idx in (("mlp.gate_proj", gi), ("mlp.up_proj", ui)):
            if (li, key) in lora.params:
                z, sc = lora.delta(x, (li, key), L.wgu[idx], training)
                if key == "mlp.gate_proj":
                    g = g + z if sc is None else (g + z) * sc
                else:
                    u = u + z if sc is None else (u + z) * sc
    if L.bgu is not None:
        g = g + L.bgu.float()[gi]
        u = u + L.bgu.float()[ui]
    if cfg.glu_epi == "geglu":
        a = Fn.gelu(g, approximate="tanh") * u
    elif cfg.glu_epi == "swiglu_oai":
        g2 = g.clamp(max=7.0)
        u2 = u.clamp(-7.0, 7.0)
        a = (u2 + 1.0) * g2 * torch.sigmoid(1.702 * g2)
    else:
        a = Fn.silu(g) * u
    return _proj_plain(L.wd, L.bd, a, lora, (li, "mlp.down_proj"), training)


def train_forward(model, tokens: torch.Tensor, lora: TrainableLoRA | None = None, training: bool = True):
    """tokens [B, S] int64 -> logits [B, S, V] fp32, differentiable in the
    LoRA parameters."""
    cfg = model.cfg
    if model.tp.world != 1:
        raise ValueError("adapter training runs with tensor-parallel world 1")
    if any(L.moe for L in model.layers):
        raise ValueError("adapter training supports dense decoders")
    B, S = tokens.shape
    dev = model.embed.device
    tokens = tokens.to(dev)
    pos = torch.arange(S, device=dev)
    cs = model.cos_sin.to(dev)
    outs = []
    for bi in range(B):
        x = model.embed[tokens[bi]].float() * cfg.embed_scale
        for li, L in enumerate(model.layers):
            h = _rms(x, L.ln1, cfg.rms_norm_eps, cfg.norm_offset_one)
            qkv = _proj_qkv(model, L, li, h, lora, training)
            qn, kn = model.H * model.D, model.KVH * model.D
            q = qkv[:, :qn].reshape(S, model.H, model.D)
            k = qkv[:, qn:qn + kn].reshape(S, model.KVH, model.D)
            v = qkv[:, qn + kn:].reshape(S, model.KVH, model.D)
            if L.q_norm is not None:
                q = _rms(q, L.q_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
                k = _rms(k, L.k_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
            q = apply_rope_ref(q, pos, cs, model.rot_dim, cfg.rope_interleaved)
            k = apply_rope_ref(k, pos, cs, model.rot_dim, cfg.rope_interleaved)
            a = attention_rows_ref(q, k, v, pos, S, cfg.scale, cfg.window(li), L.sinks, cfg.attn_logit_softcap)
            d = _proj_plain(L.wo, L.bo, a.reshape(S, -1), lora, (li, "self_attn.o_proj"), training)
            if L.post_attn_norm is not None:
                d = _rms(d, L.post_attn_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
            x = x + d
            h = _rms(x, L.ln2, cfg.rms_norm_eps, cfg.norm_offset_one)
            d = _mlp(model, L, li, h, lora, training)
            if L.post_ffn_norm is not None:
                d = _rms(d, L.post_ffn_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
            x = x + d
        h = _rms(x, model.norm, cfg.rms_norm_eps, cfg.norm_offset_one)
        lg = h @ model.lm_head.float().t()
        if cfg.final_logit_softcap > 0:
            c = cfg.final_logit_softcap
            lg = torch.tanh(lg / c) * c
        outs.append(lg)
    return torch.stack(outs)
