"""Multi-token-prediction (MTP) draft module.

Parity: the Qwen 3.5/3.6 inline MTP head (MLXLLM/Models/Qwen35MTP.swift:140-200)
and the MTP drafter protocol (MLXLMCommon/MTPDrafterModel.swift): for a
position t it fuses the target's final-normed hidden h_t with the embedding of
the token sampled at t+1,

    x = fc([rmsnorm_e(embed(tok_{t+1})), rmsnorm_h(h_t)])        fc: [H, 2H]
    y = norm(layers(x))          decoder layer(s) with their own paged KV
    logits = lm_head(y)          shared with the target; predicts tok_{t+2}

and chains k drafts by feeding y and the drafted token back in. The decoder
layers are an ordinary one-layer :class:`DecoderLM` (same kernels, own KV
cache) that shares the target's embedding and LM head.
Checkpoint names: ``mtp.pre_fc_norm_embedding``, ``mtp.pre_fc_norm_hidden``,
``mtp.fc``, ``mtp.layers.{i}.*``, ``mtp.norm``.
"""
from __future__ import annotations

import copy

import torch

from .. import ops
from .batch import ForwardBatch


class MTPModule:
    def __init__(self, target, num_layers: int = 1):
        from .decoder import DecoderLM

        tc = target.cfg
        cfg = copy.deepcopy(tc)
        cfg.num_layers = num_layers
        last_moe = tc.is_moe(tc.num_layers - 1)
        cfg.moe_layers = [last_moe] * num_layers
        cfg.layer_windows = None
        cfg.layer_types = None  # MTP layers are full-attention layers, also in hybrid models
        cfg.num_mtp_layers = 0
        self.cfg = cfg
        self.target = target
        self.inner = DecoderLM(cfg, target.device, target.dtype, tp=target.tp)
        self.fc = None
        self.norm_e = None
        self.norm_h = None

    @property
    def device(self):
        return self.inner.device

    def init_random(self, seed: int = 1, std: float = 0.02):
        m = self.inner
        m.init_random(seed, std, with_embeddings=False)
        m.embed, m.lm_head = self.target.embed, self.target.lm_head
        H = self.cfg.hidden_size
        g = torch.Generator(device=m.device).manual_seed(seed + 7919)
        self.fc = torch.empty(H, 2 * H, device=m.device, dtype=m.dtype).normal_(0.0, std, generator=g)
        one = torch.zeros if self.cfg.norm_offset_one else torch.ones
        self.norm_e = one(H, device=m.device, dtype=m.dtype)
        self.norm_h = one(H, device=m.device, dtype=m.dtype)
        return self

    def new_kv(self, max_tokens: int, kv_fp8: bool = False):
        from ..kv.paged import PagedKVCache

        return PagedKVCache.for_model(self.inner, max_tokens=max_tokens, kv_fp8=kv_fp8)

    def forward(self, fb: ForwardBatch, kv, hidden: torch.Tensor):
        """fb: the MTP positions (input_ids = the tokens at those positions);
        hidden [T, H]: the hidden of each row's previous position. Returns
        (logits [rows, V] fp32, next hidden [rows, H])."""
        cfg = self.cfg
        e = ops.embedding(fb.input_ids, self.inner.embed, cfg.embed_scale)
        xe = ops.rmsnorm(e, self.norm_e, cfg.rms_norm_eps, cfg.norm_offset_one)
        xh = ops.rmsnorm(hidden.to(e.dtype).contiguous(), self.norm_h, cfg.rms_norm_eps, cfg.norm_offset_one)
        x = ops.gemm(torch.cat([xe, xh], dim=-1).contiguous(), self.fc)
        return self.inner.forward(fb, kv, inputs_embeds=x, return_both=True)


# checkpoint layouts of MTP heads: (fc, norm_e, norm_h, final norm, layer prefix) names
#   qwen35   Qwen 3.5 / Qwen3-Next inline MTP (MLXLLM/Models/Qwen35MTP.swift:140-200)
#   deepseek DeepSeek V3 / GLM-4.5 nextn layers stored after the decoder layers
#            (layers.{N}: enorm, hnorm, eh_proj, shared_head.norm, the layer's own weights)
#   mimo     MiMo (model.mtp_layers.{i}: token_layernorm, hidden_layernorm, input_proj, final_layernorm)
def mtp_layout(tensors: dict, num_layers: int):
    """(layout name, number of MTP layers) found in a checkpoint's tensor names, or (None, 0)."""
    names = list(tensors)

    def has(sub):
        return any(sub in k for k in names)

    if has("mtp.fc.weight") or has("mtp.pre_fc_norm_embedding"):
        n = len({k.split("mtp.layers.")[1].split(".")[0] for k in names if "mtp.layers." in k})
        return "qwen35", max(n, 1)
    if has(f"layers.{num_layers}.eh_proj"):
        n = 0
        while has(f"layers.{num_layers + n}.eh_proj"):
            n += 1
        return "deepseek", n
    if has("mtp_layers.0.input_proj"):
        n = len({k.split("mtp_layers.")[1].split(".")[0] for k in names if "mtp_layers." in k})
        return "mimo", n
    return None, 0


def load_mtp(target, tensors: dict, num_layers: int | None = None) -> "MTPModule | None":
    """The MTP head stored in a checkpoint next to `target` (None when the
    checkpoint has none). Only the first MTP layer drives drafts here (the
    chained depth reuses it, as single-head checkpoints do)."""
    from ..loader.load import build_from_tensors

    L = target.cfg.num_layers
    layout, n = mtp_layout(tensors, L)
    if layout is None:
        return None

    def pick(prefix):
        out = {}
        for k, v in tensors.items():
            i = k.find(prefix)
            if i >= 0:
                out[k[i + len(prefix):]] = v
        return out

    if layout == "qwen35":
        sub = pick("mtp.")
        fc, ne, nh, fn = sub["fc.weight"], sub["pre_fc_norm_embedding.weight"], sub["pre_fc_norm_hidden.weight"], \
            sub["norm.weight"]
        layer = {k[len("layers.0."):]: v for k, v in sub.items() if k.startswith("layers.0.")}
    elif layout == "deepseek":
        sub = pick(f"layers.{L}.")
        fc, ne, nh = sub["eh_proj.weight"], sub["enorm.weight"], sub["hnorm.weight"]
        fn = sub.get("shared_head.norm.weight")
        layer = {k: v for k, v in sub.items() if not k.startswith(("eh_proj", "enorm", "hnorm", "shared_head",
                                                                       "embed_tokens"))}
    else:
        sub = pick("mtp_layers.0.")
        fc, ne, nh, fn = sub["input_proj.weight"], sub["token_layernorm.weight"], sub["hidden_layernorm.weight"], \
            sub["final_layernorm.weight"]
        layer = {k: v for k, v in sub.items() if not k.startswith(("input_proj", "token_layernorm",
                                                                       "hidden_layernorm", "final_layernorm"))}
    mod = MTPModule(target, num_layers=1)
    H = target.cfg.hidden_size
    # checkpoints whose norms are stored zero-centred (w - 1) next to the target's
    zc = 1.0 if target.cfg.extra.get("norms_zero_centred") else 0.0

    def norm(t):
        return t.float() + zc

    tens = {"embed_tokens.weight": torch.zeros(1, H), "norm.weight": norm(fn) if fn is not None else torch.ones(H)}
    tens.update({f"layers.0.{k}": (norm(v) if k.endswith("norm.weight") else v) for k, v in layer.items()})
    inner = build_from_tensors(mod.cfg, tens, target.device, target.dtype, target.tp)
    inner.embed, inner.lm_head = target.embed, target.lm_head
    mod.inner = inner
    dev, dt = target.device, target.dtype
    mod.fc = fc.to(dev, dt).contiguous()
    mod.norm_e = norm(ne).to(dev, dt)
    mod.norm_h = norm(nh).to(dev, dt)
    mod.layout, mod.checkpoint_layers = layout, n
    return mod
