"""Affine-quantised linear weights kept packed on the device.

MLX checkpoints store ``w = scale * q + bias`` per group of ``gs`` inputs with
unsigned ``bits``-bit codes packed into uint32 words (MLXNN QuantizedLinear;
layout checked at MLXLMCommon/SwitchLayers.swift:1431-1452). This module keeps
such weights packed in the layout the dequantising tcgen05 GEMM
(``b200_gemm_q``) streams:

* codes   uint8 [N, K*bits/8]. 8-bit: one code per byte, in input order.
  4-bit: each 32-bit word holds 8 consecutive inputs with input 2j in bits
  4j..4j+3 and input 2j+1 in bits 16+4j..19+4j, so one mask turns a shifted
  word into a bf16 pair (repacked once from MLX's nibble order at load).
* scales_t, biases_t  bf16 [K/gs, N] (transposed: rows of N are what a
  128-row weight tile needs, contiguous for TMA).

MXFP4 (``mode="mxfp4"``, the OCP microscaling format of GPT-OSS and MLX's
``mxfp4`` mode): 4-bit e2m1 codes (sign, two exponent bits, one mantissa bit)
in the same repacked nibble order, one power-of-two scale 2^(e8m0 - 127) per
32 inputs (kept as bf16, exact), no biases; w = e2m1(q) * scale. NVFP4
(``mode="nvfp4"``, NVIDIA ModelOpt): the same codes with one scale per 16
inputs, the e4m3 block scale times the tensor's fp32 global scale (kept as
bf16). The kernels take both as ``bits = -4`` with the group size.

Row operations used by the model builder (stacking q|k|v, interleaving
gate/up, tensor-parallel row / column shards) act on codes, scales and biases
together; groups run along K, so they commute with quantisation. Column shards
must start on a group boundary.
"""
from __future__ import annotations

import math

import torch

from . import quant

SUPPORTED_BITS = (4, 8)
# MLX affine widths the loader accepts; 2 / 3-bit codes ride in 4-bit
# records and 5 / 6-bit codes in 8-bit records (same scales and biases, so
# the dequantised values are exact)
CARRIED_BITS = {2: 4, 3: 4, 4: 4, 5: 8, 6: 8, 8: 8}
SUPPORTED_GROUPS = (32, 64, 128)  # affine / MXFP4; NVFP4 uses 16
# e2m1 magnitudes of codes 0..7 (code bit 3 is the sign)
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def e2m1_decode(q: torch.Tensor) -> torch.Tensor:
    """float values of e2m1 codes (int tensor, 0..15)."""
    lut = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=q.device)
    v = lut[(q & 7).long()]
    return torch.where((q & 8) != 0, -v, v)


def e2m1_encode(x: torch.Tensor) -> torch.Tensor:
    """Nearest e2m1 code of each value (ties to the even mantissa, saturating
    at +-6), int32."""
    a = x.abs().clamp(max=6.0)
    # midpoints between consecutive magnitudes; ties go to the code with m = 0
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=x.device)
    m = torch.bucketize(a, mids, right=False).to(torch.int32)
    # bucketize puts a value equal to a midpoint in the lower bucket; move
    # ties whose lower code is odd (m = 1) up to the even code
    tie = (a.unsqueeze(-1) == mids).any(-1) & (m % 2 == 1)
    m = torch.where(tie, m + 1, m)
    return torch.where((x < 0) & (m > 0), m | 8, m).to(torch.int32)


def e8m0_to_scale(s: torch.Tensor) -> torch.Tensor:
    """2^(s - 127) of uint8 e8m0 exponents, as float32."""
    return torch.exp2(s.to(torch.float32) - 127.0)


def _repack4(q: torch.Tensor) -> torch.Tensor:
    """int codes [N, K] (0..15) -> uint8 [N, K/2] in the kernel's nibble order."""
    N, K = q.shape
    w = q.to(torch.int32).reshape(N, K // 8, 8)
    b0 = w[..., 0] | (w[..., 2] << 4)
    b1 = w[..., 4] | (w[..., 6] << 4)
    b2 = w[..., 1] | (w[..., 3] << 4)
    b3 = w[..., 5] | (w[..., 7] << 4)
    return torch.stack([b0, b1, b2, b3], -1).reshape(N, K // 2).to(torch.uint8)


def _unpack4(c: torch.Tensor) -> torch.Tensor:
    N, KB = c.shape
    b = c.to(torch.int32).reshape(N, KB // 4, 4)
    q = torch.empty(N, KB // 4, 8, dtype=torch.int32, device=c.device)
    q[..., 0], q[..., 2] = b[..., 0] & 15, b[..., 0] >> 4
    q[..., 4], q[..., 6] = b[..., 1] & 15, b[..., 1] >> 4
    q[..., 1], q[..., 3] = b[..., 2] & 15, b[..., 2] >> 4
    q[..., 5], q[..., 7] = b[..., 3] & 15, b[..., 3] >> 4
    return q.reshape(N, KB * 2)


class QuantizedWeight:
    """Packed affine or MXFP4 weight of logical shape [N, K]."""

    def __init__(self, codes: torch.Tensor, scales_t: torch.Tensor, biases_t: torch.Tensor | None, bits: int, gs: int,
                 num_experts: int = 0, mode: str = "affine"):
        assert mode in ("affine", "mxfp4", "nvfp4")
        assert bits in SUPPORTED_BITS and (gs in SUPPORTED_GROUPS or (mode == "nvfp4" and gs == 16)), (bits, gs)
        assert mode == "affine" or (bits == 4 and gs == {"mxfp4": 32, "nvfp4": 16}[mode] and biases_t is None), \
            "e2m1 formats: 4-bit, group 32 (MXFP4) / 16 (NVFP4), no bias"
        self.codes, self.scales_t, self.biases_t = codes, scales_t, biases_t
        self.bits, self.gs, self.mode = bits, gs, mode
        self.shape = (codes.shape[0], codes.shape[1] * 8 // bits)
        # > 0: MoE experts stacked along rows, expert e owns rows [e*N/E, (e+1)*N/E)
        self.num_experts = num_experts

    @property
    def kernel_bits(self) -> int:
        """Format code of the kernels' C ABI: 4 / 8 affine, -4 MXFP4."""
        return -4 if self.mode in ("mxfp4", "nvfp4") else self.bits

    def _like(self, codes, scales_t, biases_t, num_experts: int = 0) -> "QuantizedWeight":
        return QuantizedWeight(codes, scales_t, biases_t, self.bits, self.gs, num_experts, self.mode)

    def _bsel(self, fn):
        return None if self.biases_t is None else fn(self.biases_t)

    def scaled(self, m: float) -> "QuantizedWeight":
        """The weight times `m` (affine records: scales and biases scaled;
        e2m1 records only by powers of two, else ValueError)."""
        if self.mode in ("mxfp4", "nvfp4") and not (m > 0 and math.log2(m).is_integer()):
            raise ValueError("e2m1 records scale only by powers of two")
        sc = (self.scales_t.float() * m).to(self.scales_t.dtype)
        return self._like(self.codes, sc, self._bsel(lambda b: (b.float() * m).to(b.dtype)), self.num_experts)

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_codes(cls, q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int, gs: int,
                   dtype=torch.bfloat16):
        """q int [N, K]; scales / biases [N, K/gs]."""
        codes = _repack4(q) if bits == 4 else q.to(torch.uint8).contiguous()
        return cls(codes.contiguous(), scales.t().to(dtype).contiguous(), biases.t().to(dtype).contiguous(), bits, gs)

    @classmethod
    def from_mlx(cls, packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int, gs: int):
        """MLX layout: packed uint32 (as int32) [N, K*bits/32], scales / biases
        [N, K/gs]. Widths other than 4 / 8 are stored at their carrier width."""
        K = scales.shape[-1] * gs
        q = quant.unpack_codes(packed.cpu(), bits, K)
        return cls.from_codes(q, scales.cpu(), biases.cpu(), CARRIED_BITS[bits], gs)

    @classmethod
    def from_mxfp4(cls, q: torch.Tensor, scales_e8m0: torch.Tensor):
        """e2m1 codes int [N, K] (0..15) and uint8 e8m0 exponents [N, K/32]."""
        sc = e8m0_to_scale(scales_e8m0).to(torch.bfloat16)
        return cls(_repack4(q).contiguous(), sc.t().contiguous(), None, 4, 32, mode="mxfp4")

    @classmethod
    def from_nvfp4(cls, q: torch.Tensor, block_scales: torch.Tensor, global_scale: float):
        """e2m1 codes int [N, K] and e4m3 block scales [N, K/16] (float8 or
        float) times the fp32 global scale (NVIDIA ModelOpt NVFP4)."""
        sc = (block_scales.float() * float(global_scale)).to(torch.bfloat16)
        return cls(_repack4(q).contiguous(), sc.t().contiguous(), None, 4, 16, mode="nvfp4")

    @classmethod
    def quantize_nvfp4(cls, w: torch.Tensor):
        """NVFP4 quantisation of a float weight [N, K]: global scale
        amax / (6 * 448), e4m3 block scales of amax16 / 6 / global, nearest
        e2m1 codes of w / (block * global)."""
        N, K = w.shape
        g = w.float().reshape(N, K // 16, 16)
        gscale = float(w.float().abs().max().clamp(min=1e-12)) / (6.0 * 448.0)
        bs = (g.abs().amax(-1) / 6.0 / gscale).clamp(max=448.0).to(torch.float8_e4m3fn)
        denom = (bs.float() * gscale).clamp(min=1e-30)[..., None]
        q = e2m1_encode(g / denom).reshape(N, K)
        return cls.from_nvfp4(q, bs, gscale)

    @classmethod
    def from_mlx_mxfp4(cls, packed: torch.Tensor, scales: torch.Tensor):
        """MLX ``mxfp4`` layout: uint32 words (as int32) [N, K/8], 8 codes
        per word low nibble first; uint8 scales [N, K/32]."""
        K = scales.shape[-1] * 32
        q = quant.unpack_codes(packed.cpu(), 4, K)
        return cls.from_mxfp4(q, scales.cpu())

    @classmethod
    def quantize_mxfp4(cls, w: torch.Tensor):
        """MXFP4 quantisation of a float weight [N, K] where it lives: per 32
        inputs the shared exponent floor(log2(amax)) - 2 (e2m1's largest
        exponent), then the nearest e2m1 code of w / 2^exp."""
        N, K = w.shape
        g = w.float().reshape(N, K // 32, 32)
        amax = g.abs().amax(-1, keepdim=True).clamp(min=2.0 ** -120)
        e = torch.floor(torch.log2(amax)) - 2
        s = (e + 127).clamp(0, 254)
        q = e2m1_encode(g / torch.exp2(s - 127)).reshape(N, K)
        return cls.from_mxfp4(q, s[..., 0].to(torch.uint8))

    @classmethod
    def quantize(cls, w: torch.Tensor, bits: int = 4, gs: int = 64):
        """MLX-style affine quantisation of a float weight [N, K]."""
        packed, s, b = quant.affine_quantize(w.float().cpu(), gs, bits)
        # round scale / bias to bf16 first: the kernel applies them in bf16
        return cls.from_mlx(packed, s.to(torch.bfloat16), b.to(torch.bfloat16), bits, gs)

    @classmethod
    def quantize_device(cls, w: torch.Tensor, bits: int = 4, gs: int = 64):
        """:meth:`quantize` computed where `w` lives (vectorised; for large
        random-init models on the GPU). Same rule: scale = (max - min) /
        levels, bias = min, q = round((w - bias) / scale); scale and bias are
        then stored in bf16."""
        N, K = w.shape
        g = w.float().reshape(N, K // gs, gs)
        mx = g.amax(-1, keepdim=True)
        mn = g.amin(-1, keepdim=True)
        levels = (1 << bits) - 1
        scale = ((mx - mn) / levels).clamp(min=1e-8)
        q = torch.round((g - mn) / scale).clamp(0, levels).to(torch.int32).reshape(N, K)
        codes = _repack4(q) if bits == 4 else q.to(torch.uint8)
        return cls(codes.contiguous(), scale[..., 0].t().to(torch.bfloat16).contiguous(),
                   mn[..., 0].t().to(torch.bfloat16).contiguous(), bits, gs)

    # ---------------------------------------------------------------- views
    @property
    def device(self):
        return self.codes.device

    @property
    def dtype(self):
        return self.scales_t.dtype

    def codes_int(self) -> torch.Tensor:
        return _unpack4(self.codes) if self.bits == 4 else self.codes.to(torch.int32)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        """[N, K] weights with one rounding of scale * q + bias (as the kernel);
        MXFP4: e2m1(q) * scale (exact)."""
        q = self.codes_int()
        s = self.scales_t.t().float().repeat_interleave(self.gs, dim=1)
        if self.mode in ("mxfp4", "nvfp4"):
            return (e2m1_decode(q) * s).to(torch.bfloat16).to(dtype)
        b = self.biases_t.t().float().repeat_interleave(self.gs, dim=1)
        return (q.float() * s + b).to(torch.bfloat16).to(dtype)

    def to(self, device=None, dtype=None):
        dt = dtype if dtype in (torch.bfloat16, torch.float16, torch.float32) else None
        if self.mode in ("mxfp4", "nvfp4"):
            dt = None  # block scales stay bf16
        sc = self.scales_t.to(device=device, dtype=dt or self.scales_t.dtype)
        bi = self._bsel(lambda b: b.to(device=device, dtype=dt or b.dtype))
        return self._like(self.codes.to(device), sc, bi, self.num_experts)

    def select_rows(self, idx: torch.Tensor, num_experts: int = 0) -> "QuantizedWeight":
        """Rows `idx` (any order) as a new weight."""
        idx = idx.to(self.codes.device)
        return self._like(self.codes.index_select(0, idx).contiguous(), self.scales_t.index_select(1, idx).contiguous(),
                          self._bsel(lambda b: b.index_select(1, idx).contiguous()), num_experts)

    @staticmethod
    def stack_experts(parts: list["QuantizedWeight"]) -> "QuantizedWeight":
        """Experts [E] of shape [N, K] -> one weight [E*N, K] with num_experts = E."""
        w = QuantizedWeight.cat_rows(parts)
        w.num_experts = len(parts)
        return w

    def expert(self, e: int) -> "QuantizedWeight":
        n = self.shape[0] // self.num_experts
        return self.rows(e * n, (e + 1) * n)

    # ---------------------------------------------------------------- device layout
    def record_bytes(self) -> int:
        gpb = {16: 4, 32: 2}.get(self.gs, 1)
        return self.bits * 128 * 8 + gpb * (256 if self.biases_t is None else 512)

    def tiled_natural(self) -> torch.Tensor:
        """e2m1 records with the codes in natural order (input 2j in the low
        nibble of byte j, 2j+1 in the high nibble): the layout the hardware
        pair conversion of the f16 MoE path reads (built once, cached)."""
        t = getattr(self, "_tiled_nat", None)
        if t is None:
            assert self.kernel_bits == -4, "natural-order records are for e2m1 codes"
            q = _unpack4(self.codes)
            nat = (q[:, 0::2] | (q[:, 1::2] << 4)).to(torch.uint8).contiguous()
            t = self._tiled_nat = self.tiled(codes=nat, cache=False)
        return t

    def f16_scales_ok(self) -> bool:
        """Every e2m1 weight times its block scale is a normal f16 (scales in
        [2^-14, 2^13]): the f16 MoE path is exact then."""
        ok = getattr(self, "_f16_ok", None)
        if ok is None:
            sc = self.scales_t.float().abs()
            nz = sc[sc > 0]
            ok = self._f16_ok = bool(sc.numel() == 0 or (nz.numel() == 0 or (nz.min() >= 2.0 ** -14
                                                                           and sc.max() <= 2.0 ** 13)))
        return ok

    def tiled(self, codes: torch.Tensor | None = None, cache: bool = True) -> torch.Tensor:
        """Tile-major device layout streamed by the dequantising kernels
        (built once, cached): for each 128-row tile (per expert when experts
        are stacked; rows past the end are zero) and each 64-input K block one
        contiguous record {codes [128][bits*8 B], scales [gpb][128] bf16,
        biases [gpb][128] bf16}; gpb = 2 for group size 32, else 1 (a
        128-input group repeats its scale and bias in both of its blocks)."""
        t = getattr(self, "_tiled", None) if cache else None
        if t is not None:
            return t
        E = self.num_experts or 1
        N, K = self.shape
        Ne = N // E
        tiles = (Ne + 127) // 128
        KB = K // 64
        cb = self.bits * 8  # code bytes per row per K block
        dev = self.codes.device
        codes = (self.codes if codes is None else codes).view(E, Ne, KB, cb)
        sc = self.scales_t.t().reshape(E, Ne, -1)  # [E, Ne, G]
        bi = self.biases_t.t().reshape(E, Ne, -1) if self.biases_t is not None else torch.zeros_like(sc)
        pad = tiles * 128 - Ne
        if pad:
            codes = torch.cat([codes, torch.zeros(E, pad, KB, cb, dtype=codes.dtype, device=dev)], 1)
            sc = torch.cat([sc, torch.zeros(E, pad, sc.shape[2], dtype=sc.dtype, device=dev)], 1)
            bi = torch.cat([bi, torch.zeros(E, pad, bi.shape[2], dtype=bi.dtype, device=dev)], 1)
        if self.gs in (16, 32):  # groups of each K block: [E, rows, KB, gpb]
            gpb = 64 // self.gs
            sc_kb, bi_kb = sc.reshape(E, -1, KB, gpb), bi.reshape(E, -1, KB, gpb)
        elif self.gs == 64:
            sc_kb, bi_kb = sc.reshape(E, -1, KB, 1), bi.reshape(E, -1, KB, 1)
        else:  # 128: one group per two K blocks
            sc_kb = sc.repeat_interleave(2, dim=2).reshape(E, -1, KB, 1)
            bi_kb = bi.repeat_interleave(2, dim=2).reshape(E, -1, KB, 1)
        c = codes.reshape(E, tiles, 128, KB, cb).permute(0, 1, 3, 2, 4).reshape(E, tiles, KB, 128 * cb)
        s_ = sc_kb.reshape(E, tiles, 128, KB, -1).permute(0, 1, 3, 4, 2).contiguous()  # [E, t, KB, gpb, 128]
        b_ = bi_kb.reshape(E, tiles, 128, KB, -1).permute(0, 1, 3, 4, 2).contiguous()
        s_b = s_.view(torch.uint8).reshape(E, tiles, KB, -1)
        b_b = b_.view(torch.uint8).reshape(E, tiles, KB, -1)
        rec = torch.cat([c, s_b] if self.biases_t is None else [c, s_b, b_b], dim=-1).contiguous()
        assert rec.shape[-1] == self.record_bytes()
        rec = rec.reshape(-1)
        if cache:
            self._tiled = rec
        return rec

    def numel(self) -> int:
        return self.shape[0] * self.shape[1]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.codes, self.scales_t, self.biases_t) if t is not None)

    # ---------------------------------------------------------------- row / column ops
    def rows(self, lo: int, hi: int) -> "QuantizedWeight":
        return self._like(self.codes[lo:hi].contiguous(), self.scales_t[:, lo:hi].contiguous(),
                          self._bsel(lambda b: b[:, lo:hi].contiguous()))

    def cols(self, lo: int, hi: int) -> "QuantizedWeight":
        assert lo % self.gs == 0 and hi % self.gs == 0, "column shards must align with quantisation groups"
        c0, c1 = lo * self.bits // 8, hi * self.bits // 8
        g0, g1 = lo // self.gs, hi // self.gs
        return self._like(self.codes[:, c0:c1].contiguous(), self.scales_t[g0:g1].contiguous(),
                          self._bsel(lambda b: b[g0:g1].contiguous()))

    @staticmethod
    def cat_rows(parts: list["QuantizedWeight"]) -> "QuantizedWeight":
        p0 = parts[0]
        assert all(p.bits == p0.bits and p.gs == p0.gs and p.mode == p0.mode for p in parts)
        bi = None if p0.biases_t is None else torch.cat([p.biases_t for p in parts], 1)
        return p0._like(torch.cat([p.codes for p in parts], 0), torch.cat([p.scales_t for p in parts], 1), bi)

    @staticmethod
    def interleave_gate_up(g: "QuantizedWeight", u: "QuantizedWeight", block: int = 64) -> "QuantizedWeight":
        F = g.shape[0]
        assert F % block == 0 and u.shape == g.shape
        idx = []
        for b in range(F // block):
            idx.append(("g", b))
            idx.append(("u", b))
        parts = [(g if w == "g" else u).rows(b * block, (b + 1) * block) for w, b in idx]
        return QuantizedWeight.cat_rows(parts)


def is_quantized(w) -> bool:
    return isinstance(w, QuantizedWeight)
