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
