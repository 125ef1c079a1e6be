"""Batched multi-adapter LoRA ops (``csrc/kernels/lora.cu``) and their fp32
CPU statements.

Per adapted projection with stacked adapters A [S, R, K] and B^T [S, R, N]:
``lora_shrink`` t = A[slot] x (fp32 [T, R]); ``lora_expand`` y += c[slot] *
t B^T[slot] in place; ``lora_expand_glu`` adds the delta to an interleaved
gate|up pre-activation and applies the gated activation. Rows with a negative
slot carry no adapter.
"""
from __future__ import annotations

import torch

from . import _lib
from .reference import deinterleave_gate_up

GLU_CODES = {"swiglu": 1, "geglu": 4, "swiglu_oai": 5}


def _glu_ref(g, u, act):
    if act == "geglu":
        return torch.nn.functional.gelu(g, approximate="tanh") * u
    if act == "swiglu_oai":
        g = g.clamp(max=7.0)
        u = u.clamp(-7.0, 7.0)
        return (u + 1.0) * g * torch.sigmoid(1.702 * g)
    return torch.nn.functional.silu(g) * u


def lora_shrink(x: torch.Tensor, A: torch.Tensor, slots: torch.Tensor, out: torch.Tensor | None = None):
    T, K = x.shape
    S, R, _ = A.shape
    if out is None:
        out = torch.empty(T, R, dtype=torch.float32, device=x.device)
    if not x.is_cuda:
        s = slots.long()
        ok = (s >= 0) & (s < S)
        t = torch.zeros(T, R, dtype=torch.float32)
        if ok.any():
            t[ok] = torch.einsum("trk,tk->tr", A[s[ok]].float(), x[ok].float())
        out.copy_(t)
        return out
    if x.stride(1) != 1:
        x = x.contiguous()
    rc = _lib.lib().b200_lora_shrink(x.data_ptr(), x.stride(0), A.data_ptr(), R, K, slots.data_ptr(), S,
                                     out.data_ptr(), T, _lib.stream_ptr(x.device))
    _lib.check(rc, f"lora_shrink T={T} R={R} K={K}")
    _lib.count(1)
    return out


def lora_expand(y: torch.Tensor, Bt: torch.Tensor, t: torch.Tensor, slots: torch.Tensor, scale: torch.Tensor):
    """y [T, N] += scale[slot] * t @ Bt[slot] (rounded to y's dtype), in place."""
    T, N = y.shape
    S, R, _ = Bt.shape
    if not y.is_cuda:
        s = slots.long()
        ok = (s >= 0) & (s < S)
        if ok.any():
            d = torch.einsum("tr,trn->tn", t[ok].float(), Bt[s[ok]].float()) * scale[s[ok]].float()[:, None]
            y[ok] = (y[ok].float() + d).to(y.dtype)
        return y
    rc = _lib.lib().b200_lora_expand(y.data_ptr(), y.stride(0), Bt.data_ptr(), R, N, t.data_ptr(), slots.data_ptr(),
                                     scale.data_ptr(), S, T, _lib.stream_ptr(y.device))
    _lib.check(rc, f"lora_expand T={T} R={R} N={N}")
    _lib.count(1)
    return y


def lora_expand_glu(gu: torch.Tensor, Bt: torch.Tensor, t: torch.Tensor, slots: torch.Tensor, scale: torch.Tensor,
                    act: str = "swiglu", out: torch.Tensor | None = None):
    """gu [T, 2F] interleaved gate|up pre-activation (64-row blocks) plus the
    adapter delta, then the gated activation: [T, F]."""
    T, F2 = gu.shape
    F = F2 // 2
    S, R, _ = Bt.shape
    if out is None:
        out = torch.empty(T, F, dtype=gu.dtype, device=gu.device)
    if not gu.is_cuda:
        pre = gu.float()
        s = slots.long()
        ok = (s >= 0) & (s < S)
        if ok.any():
            d = torch.einsum("tr,trn->tn", t[ok].float(), Bt[s[ok]].float()) * scale[s[ok]].float()[:, None]
            pre = pre.clone()
            pre[ok] = (pre[ok] + d).to(gu.dtype).float()
        g, u = deinterleave_gate_up(pre.t())
        out.copy_(_glu_ref(g.t(), u.t(), act).to(gu.dtype))
        return out
    rc = _lib.lib().b200_lora_expand_glu(gu.data_ptr(), gu.stride(0), out.data_ptr(), out.stride(0), F, Bt.data_ptr(),
                                         R, t.data_ptr(), slots.data_ptr(), scale.data_ptr(), S, GLU_CODES[act], T,
                                         _lib.stream_ptr(gu.device))
    _lib.check(rc, f"lora_expand_glu T={T} R={R} F={F}")
    _lib.count(1)
    return out
