"""Quantise a built model's weights in place to MLX-style affine codes kept
packed on the device (:class:`QuantizedWeight`), e.g. to run a random-init
model in the quantised serving configuration of a checkpoint.

Parity: MLXLMCommon quantize (``quantize(model:groupSize:bits:)`` with a
per-layer predicate), applied here to the fused projection layouts: dense
projections (q|k|v, o, gate/up, down), MoE expert stacks (gate/up, down) and,
optionally, the LM head. Embedding tables stay bf16 (rows are gathered).
"""
from __future__ import annotations

import torch

from ..ops.qlinear import QuantizedWeight


def _q(t: torch.Tensor, bits: int, gs: int, device, mode: str = "affine") -> QuantizedWeight:
    if mode == "mxfp4":
        return QuantizedWeight.quantize_mxfp4(t).to(device)
    return QuantizedWeight.quantize_device(t, bits, gs).to(device)


def quantize_model(model, bits: int = 4, group_size: int = 64, dense: bool = True, experts: bool = True,
                   lm_head: bool = False, mode: str = "affine"):
    """`mode="mxfp4"`: OCP MXFP4 (e2m1 codes, e8m0 scale per 32 inputs; the
    GPT-OSS expert format); `bits` / `group_size` are then 4 / 32."""
    if mode == "mxfp4":
        bits, group_size = 4, 32
    for L in model.layers:
        quantize_layer(L, model.device, bits, group_size, dense, experts, mode)
    if lm_head and isinstance(model.lm_head, torch.Tensor) and model.lm_head is not model.embed:
        model.lm_head = _q(model.lm_head, bits, group_size, model.device, mode)
    return model


def quantize_layer(L, dev, bits: int = 4, group_size: int = 64, dense: bool = True, experts: bool = True,
                   mode: str = "affine"):
    """Quantise one layer's matrices in place (the per-layer step of
    :func:`quantize_model`; also the ``layer_hook`` of ``init_random`` for
    models whose bf16 expert weights would not fit on the device at once)."""
    if mode == "mxfp4":
        bits, group_size = 4, 32
    if dense:
        for name in ("wqkv", "wo", "wgu", "wd", "shared_gu", "shared_d"):
            t = getattr(L, name)
            if isinstance(t, torch.Tensor) and t.shape[1] % group_size == 0 and t.shape[0] % 8 == 0:
                setattr(L, name, _q(t, bits, group_size, dev, mode))
    if experts and L.moe and isinstance(L.experts_gu, torch.Tensor):
        # all experts at once: groups run along K, so quantising the
        # stacked [E*N, K] matrix equals quantising each expert
        E = L.experts_gu.shape[0]
        L.experts_gu = _q(L.experts_gu.reshape(-1, L.experts_gu.shape[-1]), bits, group_size, dev, mode)
        L.experts_gu.num_experts = E
        L.experts_d = _q(L.experts_d.reshape(-1, L.experts_d.shape[-1]), bits, group_size, dev, mode)
        L.experts_d.num_experts = E
    return L
