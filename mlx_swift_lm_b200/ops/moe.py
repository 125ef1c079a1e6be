"""MoE expert computation (sort tokens by expert -> per-expert GLU MLP ->
weighted un-sort), the SwitchGLU of MLXLMCommon/SwitchLayers.swift:478
(gatherSort :244, scatterUnsort :257, weightedExpertUnsort :149).

On CUDA the grouped path runs the fused grouped-GEMM kernels of
``csrc/kernels/moe.cu`` when they are built in; otherwise each expert's rows go
through the dense tcgen05 GEMM.
"""
from __future__ import annotations

import torch

from . import _lib
from .linear import gemm


def route_topk(logits: torch.Tensor, k: int, mode: str = "softmax_topk", norm_topk: bool = True):
    """Router top-k. softmax_topk: softmax over experts then top-k (optionally
    renormalised); topk_softmax: top-k logits then softmax over the k."""
    if mode == "topk_softmax":
        v, idx = torch.topk(logits.float(), k, dim=-1)
        return torch.softmax(v, dim=-1), idx
    p = torch.softmax(logits.float(), dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True)
    return w, idx


def moe_experts(h, experts_gu, experts_d, w, idx, epi="swiglu", gu_bias=None, d_bias=None):
    """h [T, K]; experts_gu [E, 2F, K] (64-row interleaved gate/up); experts_d [E, K, F];
    w [T, k] fp32 weights; idx [T, k] expert ids. Returns [T, K] in h.dtype."""
    T, K = h.shape
    k = idx.shape[1]
    flat = idx.reshape(-1)
    order = torch.argsort(flat, stable=True)
    tok = order // k
    wsorted = w.reshape(-1)[order]
    counts = torch.bincount(flat, minlength=experts_gu.shape[0]).tolist()
    out = torch.zeros((T, K), dtype=torch.float32, device=h.device)
    start = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        rows = tok[start:start + c]
        x = h.index_select(0, rows).contiguous()
        gu = gemm(x, experts_gu[e], epi=epi, bias=None if gu_bias is None else gu_bias[e])
        y = gemm(gu, experts_d[e], bias=None if d_bias is None else d_bias[e])
        out.index_add_(0, rows, y.float() * wsorted[start:start + c, None])
        start += c
    return out.to(h.dtype)


_ = _lib  # kernels registered by moe.cu bindings when present
