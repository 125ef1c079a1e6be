"""Gated DeltaNet (linear attention) op: conv + gates + delta-rule recurrence
+ gated RMSNorm over a flattened batch of rows, on the kernels of
``csrc/kernels/gdn.cu`` for CUDA tensors and the fp32 oracle
(:func:`reference.gdn_layer_ref`) for CPU tensors.

Parity: MLXLMCommon/GatedDelta.swift (gated_delta_step) and the GDN block of
MLXLLM/Models/Qwen3Next.swift:165-415 / Qwen35.swift:255.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from . import reference as ref

_lib.register_signatures({
    "b200_gdn_conv": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.vp, _lib.vp, _lib.vp,
                                 _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.vp, _lib.f32,
                                 _lib.vp, _lib.vp, _lib.i32, _lib.vp, _lib.f32, _lib.f32, _lib.vp]),
    "b200_gdn_recurrence": (_lib.i32, [_lib.vp, _lib.vp, _lib.vp, _lib.i32, _lib.vp, _lib.vp, _lib.vp, _lib.i32,
                                       _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.vp, _lib.i32, _lib.vp, _lib.i32,
                                       _lib.i32, _lib.i32, _lib.vp, _lib.vp]),
    "b200_group_norm_gate": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.f32,
                                        _lib.vp, _lib.i32, _lib.vp]),
    "b200_gdn_norm_gate": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.f32,
                                      _lib.vp, _lib.i32, _lib.vp]),
    "b200_short_conv": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.vp, _lib.vp,
                                   _lib.vp, _lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp]),
    "b200_sigmoid_mul": (_lib.i32, [_lib.vp, _lib.i32, _lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.i32,
                                    _lib.vp]),
}, status_tags=("gdn",))


@dataclass
class GdnRows:
    """Rows of a forward batch as the recurrent layers see them: tokens
    cu[r]..cu[r+1]-1, state slot, and whether the row starts at position 0."""
    cu: torch.Tensor  # [R+1] int32
    fresh: torch.Tensor  # [R] int32
    slot: torch.Tensor  # [R] int32
    cu_host: list | None = None

    @property
    def num_rows(self) -> int:
        return int(self.slot.shape[0])


def gdn_layer(P: torch.Tensor, rows: GdnRows, conv_state: torch.Tensor, ssm_state: torch.Tensor,
              conv_w: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor, norm_w: torch.Tensor, Hk: int, Dk: int,
              Hv: int, Dv: int, eps: float) -> torch.Tensor:
    """P [T, C + Hv*Dv + 2*Hv] (q|k|v|z|b|a rows of the fused in-projection);
    returns the gated-normalised output [T, Hv*Dv] (input of out_proj) and
    advances each row's conv / recurrent state."""
    T = P.shape[0]
    C = 2 * Hk * Dk + Hv * Dv
    if not P.is_cuda:
        cu = rows.cu_host if rows.cu_host is not None else rows.cu.tolist()
        return ref.gdn_layer_ref(P, cu, rows.fresh.tolist(), rows.slot.tolist(), conv_state, ssm_state, conv_w, A_log,
                                 dt_bias, norm_w, Hk, Dk, Hv, Dv, eps)
    L = _lib.lib()
    st = _lib.stream_ptr(P.device)
    R = rows.num_rows
    qkv = torch.empty(T, C, dtype=torch.float32, device=P.device)
    gb = torch.empty(T, 2 * Hv, dtype=torch.float32, device=P.device)
    o = torch.empty(T, Hv * Dv, dtype=torch.float32, device=P.device)
    y = torch.empty(T, Hv * Dv, dtype=P.dtype, device=P.device)
    _lib.check(L.b200_gdn_conv(P.data_ptr(), P.stride(0), T, rows.cu.data_ptr(), R, rows.fresh.data_ptr(),
                               rows.slot.data_ptr(), conv_state.data_ptr(), conv_w.data_ptr(), C, Hk, Dk, Hv, Dv,
                               A_log.data_ptr(), dt_bias.data_ptr(), float(eps), qkv.data_ptr(), gb.data_ptr(), 0,
                               None, 0.0, 0.0, st), "gdn_conv")
    _lib.check(L.b200_gdn_recurrence(qkv.data_ptr(), gb.data_ptr(), rows.cu.data_ptr(), R, rows.fresh.data_ptr(),
                                     rows.slot.data_ptr(), ssm_state.data_ptr(), Hk, Dk, Hv, Dv, o.data_ptr(),
                                     P.data_ptr(), P.stride(0), conv_state.data_ptr(), C, T, 0, None, st),
               "gdn_recurrence")
    _lib.check(L.b200_gdn_norm_gate(o.data_ptr(), T, Hv, Dv, P[:, C:].data_ptr(), P.stride(0), norm_w.data_ptr(),
                                    float(eps), y.data_ptr(), y.stride(0), st), "gdn_norm_gate")
    _lib.count(3)
    return y


def mamba_layer(P: torch.Tensor, rows: GdnRows, conv_state: torch.Tensor, ssm_state: torch.Tensor,
                conv_w: torch.Tensor, conv_b: torch.Tensor | None, A_log: torch.Tensor, dt_bias: torch.Tensor,
                D: torch.Tensor, norm_w: torch.Tensor, G: int, N: int, H: int, Pd: int, eps: float, norm_group: int,
                dt_limits: tuple[float, float] = (0.0, float("inf"))) -> torch.Tensor:
    """Mamba-2 mixer body. P [T, C + H*Pd + H] = C | B | x (the conv
    channels, C = 2*G*N + H*Pd) | z | dt rows of the fused in-projection;
    returns rmsnorm_groups(y * silu(z)) * norm_w [T, H*Pd] (input of
    out_proj) and advances each row's conv / SSM state ([S, H, Pd, N] fp32).
    Parity: MLXLLM/Models/SSM.swift (computeDt, the SSM step) and
    MLXLLM/Models/NemotronH.swift:51-160 (conv + SiLU, gated group norm)."""
    T = P.shape[0]
    C = 2 * G * N + H * Pd
    if not P.is_cuda:
        cu = rows.cu_host if rows.cu_host is not None else rows.cu.tolist()
        return ref.mamba_layer_ref(P, cu, rows.fresh.tolist(), rows.slot.tolist(), conv_state, ssm_state, conv_w,
                                   conv_b, A_log, dt_bias, D, norm_w, G, N, H, Pd, eps, norm_group, dt_limits)
    L = _lib.lib()
    st = _lib.stream_ptr(P.device)
    R = rows.num_rows
    xbc = torch.empty(T, C, dtype=torch.float32, device=P.device)
    gb = torch.empty(T, 2 * H, dtype=torch.float32, device=P.device)
    o = torch.empty(T, H * Pd, dtype=torch.float32, device=P.device)
    y = torch.empty(T, H * Pd, dtype=P.dtype, device=P.device)
    tmin, tmax = float(dt_limits[0]), float(min(dt_limits[1], 3.0e38))
    _lib.check(L.b200_gdn_conv(P.data_ptr(), P.stride(0), T, rows.cu.data_ptr(), R, rows.fresh.data_ptr(),
                               rows.slot.data_ptr(), conv_state.data_ptr(), conv_w.data_ptr(), C, G, N, H, Pd,
                               A_log.data_ptr(), dt_bias.data_ptr(), float(eps), xbc.data_ptr(), gb.data_ptr(), 1,
                               _lib.ptr(conv_b), tmin, tmax, st), "mamba_conv")
    _lib.check(L.b200_gdn_recurrence(xbc.data_ptr(), gb.data_ptr(), rows.cu.data_ptr(), R, rows.fresh.data_ptr(),
                                     rows.slot.data_ptr(), ssm_state.data_ptr(), G, N, H, Pd, o.data_ptr(),
                                     P.data_ptr(), P.stride(0), conv_state.data_ptr(), C, T, 1, D.data_ptr(), st),
               "mamba_recurrence")
    _lib.check(L.b200_group_norm_gate(o.data_ptr(), T, H * Pd, norm_group, P[:, C:].data_ptr(), P.stride(0),
                                      norm_w.data_ptr(), float(eps), y.data_ptr(), y.stride(0), st), "mamba_norm")
    _lib.count(3)
    return y


def short_conv(P: torch.Tensor, rows: GdnRows, conv_state: torch.Tensor, conv_w: torch.Tensor,
               conv_b: torch.Tensor | None) -> torch.Tensor:
    """LFM2 short convolution: P [T, 3C] = B | C | x rows of the in-projection;
    returns C * conv(B * x) [T, C] (input of out_proj) and advances each
    row's conv state [S, taps-1, C] (the last Bx values).
    Parity: MLXLLM/Models/LFM2.swift:207-233."""
    T = P.shape[0]
    C = conv_w.shape[0]
    taps = conv_w.shape[1]
    if not P.is_cuda:
        cu = rows.cu_host if rows.cu_host is not None else rows.cu.tolist()
        return ref.short_conv_ref(P, cu, rows.fresh.tolist(), rows.slot.tolist(), conv_state, conv_w, conv_b)
    out = torch.empty(T, C, dtype=P.dtype, device=P.device)
    _lib.check(_lib.lib().b200_short_conv(P.data_ptr(), P.stride(0), T, rows.cu.data_ptr(), rows.num_rows,
                                          rows.fresh.data_ptr(), rows.slot.data_ptr(), conv_state.data_ptr(),
                                          conv_w.data_ptr(), _lib.ptr(conv_b), C, taps, out.data_ptr(),
                                          out.stride(0), _lib.stream_ptr(P.device)), "short_conv")
    _lib.count(2)
    return out


def sigmoid_mul(x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """x * sigmoid(g) (the output gate of gated attention), in x.dtype."""
    if not x.is_cuda:
        return (x.float() * torch.sigmoid(g.float())).to(x.dtype)
    T, N = x.shape
    out = torch.empty(T, N, dtype=x.dtype, device=x.device)
    _lib.check(_lib.lib().b200_sigmoid_mul(x.data_ptr(), x.stride(0), g.data_ptr(), g.stride(0), T, N, out.data_ptr(),
                                           out.stride(0), _lib.stream_ptr(x.device)), "sigmoid_mul")
    _lib.count(1)
    return out
