"""Quantized weight formats of MLX checkpoints (CPU reference codecs).

* affine (``mode: affine``): per group of ``group_size`` input columns,
  ``w = scale * q + bias`` with unsigned ``bits``-bit codes packed little-end
  first into uint32 words (``weight`` [out, in*bits/32], ``scales`` and
  ``biases`` [out, in/group_size]); layout checked by the reference at
  MLXLMCommon/SwitchLayers.swift:1431-1452, config BaseConfiguration.swift:22-68.
* ``mxfp4``: e2m1 codes (8 per uint32), one e8m0 scale byte per 32 inputs.
* ``nvfp4``: e2m1 codes, one fp8-e4m3 scale per 16 inputs.
* ``mxfp8``: fp8-e4m3 codes, one e8m0 scale per 32 inputs.

These codecs define the semantics the dequantising GEMV/GEMM kernels match.
"""
from __future__ import annotations

import numpy as np
import torch

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def unpack_codes(packed: torch.Tensor, bits: int, n: int) -> torch.Tensor:
    """uint32-packed (stored as int32) [R, n*bits/32] -> int64 codes [R, n]."""
    p = packed.to(torch.int64) & 0xFFFFFFFF
    per = 32 // bits
    if 32 % bits == 0:
        shifts = torch.arange(per, dtype=torch.int64) * bits
        codes = (p[..., :, None] >> shifts) & ((1 << bits) - 1)
        return codes.reshape(*packed.shape[:-1], -1)[..., :n]
    # bit-stream packing for 3/5/6 bits
    R = p.shape[:-1]
    words = p.reshape(-1, p.shape[-1]).numpy().astype(np.uint64)
    out = np.zeros((words.shape[0], n), np.int64)
    for i in range(n):
        bit = i * bits
        w, o = divmod(bit, 32)
        v = words[:, w] >> np.uint64(o)
        if o + bits > 32:
            v |= words[:, w + 1] << np.uint64(32 - o)
        out[:, i] = (v & np.uint64((1 << bits) - 1)).astype(np.int64)
    return torch.from_numpy(out).reshape(*R, n)


def pack_codes(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """int codes [R, n] -> uint32 words stored as int32 [R, n*bits/32]."""
    c = codes.to(torch.int64)
    n = c.shape[-1]
    if 32 % bits == 0:
        per = 32 // bits
        c = c.reshape(*c.shape[:-1], n // per, per)
        shifts = torch.arange(per, dtype=torch.int64) * bits
        w = (c << shifts).sum(-1)
        return torch.from_numpy((w & 0xFFFFFFFF).numpy().astype(np.uint32).view(np.int32))
    R = c.shape[:-1]
    cc = c.reshape(-1, n).numpy().astype(np.uint64)
    nw = (n * bits + 31) // 32
    words = np.zeros((cc.shape[0], nw), np.uint64)
    for i in range(n):
        bit = i * bits
        w, o = divmod(bit, 32)
        words[:, w] |= (cc[:, i] << np.uint64(o)) & np.uint64(0xFFFFFFFF)
        if o + bits > 32:
            words[:, w + 1] |= cc[:, i] >> np.uint64(32 - o)
    return torch.from_numpy(words.astype(np.uint32).view(np.int32)).reshape(*R, nw)


def affine_quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """MLX-style affine quantisation: returns (packed int32, scales, biases)."""
    out, inn = w.shape
    g = w.float().reshape(out, inn // group_size, group_size)
    mx = g.amax(-1, keepdim=True)
    mn = g.amin(-1, keepdim=True)
    levels = (1 << bits) - 1
    scale = ((mx - mn) / levels).clamp(min=1e-8)
    bias = mn
    q = torch.round((g - bias) / scale).clamp(0, levels).to(torch.int64).reshape(out, inn)
    return pack_codes(q, bits), scale[..., 0], bias[..., 0]


def affine_dequantize(packed, scales, biases, group_size: int = 64, bits: int = 4, dtype=torch.float32):
    out = scales.shape[0]
    inn = scales.shape[-1] * group_size
    q = unpack_codes(packed.cpu(), bits, inn).float().reshape(*scales.shape, group_size)
    w = q * scales.cpu().float()[..., None] + biases.cpu().float()[..., None]
    return w.reshape(*scales.shape[:-1], inn).to(dtype)


def e8m0_to_float(s: torch.Tensor) -> torch.Tensor:
    return torch.pow(2.0, s.to(torch.int64).float() - 127.0)


def mxfp4_dequantize(packed, scales, group_size: int = 32, dtype=torch.float32):
    inn = scales.shape[-1] * group_size
    codes = unpack_codes(packed.cpu(), 4, inn)
    v = E2M1[codes]
    sc = e8m0_to_float(scales.cpu().to(torch.int64) & 0xFF)
    return (v.reshape(*scales.shape, group_size) * sc[..., None]).reshape(*scales.shape[:-1], inn).to(dtype)


def mxfp4_quantize(w: torch.Tensor, group_size: int = 32):
    """Round-to-nearest MXFP4 (e2m1 codes, e8m0 scales)."""
    out, inn = w.shape
    g = w.float().reshape(out, inn // group_size, group_size)
    amax = g.abs().amax(-1).clamp(min=1e-30)
    e = torch.floor(torch.log2(amax)) - 2  # largest e2m1 magnitude is 6 = 1.5 * 2^2
    e = e.clamp(-127, 127)
    sc = torch.pow(2.0, e)
    x = g / sc[..., None]
    mags = E2M1[:8]
    idx = (x.abs()[..., None] - mags).abs().argmin(-1)
    codes = idx + (x < 0).to(torch.int64) * 8
    codes = torch.where(idx == 0, torch.zeros_like(codes), codes)
    return pack_codes(codes.reshape(out, inn), 4), (e + 127).to(torch.uint8)


def nvfp4_dequantize(packed, scales, group_size: int = 16, global_scale: float = 1.0, dtype=torch.float32):
    inn = scales.shape[-1] * group_size
    codes = unpack_codes(packed.cpu(), 4, inn)
    v = E2M1[codes]
    sc = scales.cpu().view(torch.float8_e4m3fn).float() if scales.dtype == torch.uint8 else scales.cpu().float()
    return (v.reshape(*scales.shape, group_size) * sc[..., None] * global_scale).reshape(
        *scales.shape[:-1], inn).to(dtype)


def mxfp8_dequantize(weight, scales, group_size: int = 32, dtype=torch.float32):
    inn = scales.shape[-1] * group_size
    v = weight.cpu().view(torch.float8_e4m3fn).float() if weight.dtype == torch.uint8 else weight.cpu().float()
    sc = e8m0_to_float(scales.cpu().to(torch.int64) & 0xFF)
    return (v.reshape(*scales.shape, group_size) * sc[..., None]).reshape(*scales.shape[:-1], inn).to(dtype)


def dequantize(weight, scales, biases=None, mode: str = "affine", group_size: int = 64, bits: int = 4,
               dtype=torch.float32):
    if mode == "affine":
        return affine_dequantize(weight, scales, biases, group_size, bits, dtype)
    if mode == "mxfp4":
        return mxfp4_dequantize(weight, scales, group_size or 32, dtype)
    if mode == "nvfp4":
        return nvfp4_dequantize(weight, scales, group_size or 16, 1.0, dtype)
    if mode == "mxfp8":
        return mxfp8_dequantize(weight, scales, group_size or 32, dtype)
    raise ValueError(f"unknown quantization mode {mode}")
