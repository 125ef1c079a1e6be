"""Activation transforms before quantised linears: ParoQuant pairwise
rotations and Prism block-Hadamard transforms.

Parity: MLXLMCommon/ParoQuant (RotateQuantizedLinear.swift:10-80 - y =
quantised_matmul(rotate(x), W); PairwiseRotation.swift - channel scales then
`krot` rounds of Givens rotations of disjoint channel pairs inside each
128-channel group; RotateSwitchGLU.swift - experts share one rotation per
projection and layer; ParoQuantLoader.swift - AutoAWQ packing).

:class:`PairwiseRotation` holds one rotation (cos / sin / packed pairs per
round, channel scales); ``rotate`` runs ``b200_pair_rotate``
(csrc/kernels/rotation.cu) on CUDA and the fp32 re-statement on CPU.
:class:`RotatedWeight` is a weight ``ops.gemm`` accepts: row blocks, each
with its own rotation and (quantised) weight, so fused projections (q|k|v,
gate/up) keep working when their parts were rotated differently.
"""
from __future__ import annotations

import torch

from . import _lib

_lib.register_signatures({
    "b200_pair_rotate": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.vp, _lib.vp, _lib.vp,
                                    _lib.i32, _lib.vp, _lib.i32, _lib.vp]),
    "b200_block_hadamard": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp,
                                       _lib.i32, _lib.vp]),
}, status_tags=("rotation",))

GROUP = 128


class PairwiseRotation:
    def __init__(self, theta: torch.Tensor, pairs: torch.Tensor, channel_scales: torch.Tensor | None = None):
        """theta [krot, K/2] angles; pairs [krot, K] local channel indices
        (even / odd entries of each group form the pairs); channel_scales [K]."""
        krot, K = pairs.shape
        assert K % GROUP == 0 and theta.shape == (krot, K // 2)
        th = theta.float()
        self.cos, self.sin = th.cos().contiguous(), th.sin().contiguous()
        p = pairs.to(torch.int32).reshape(krot, K // GROUP, GROUP)
        self.pairs = (p[..., 0::2] | (p[..., 1::2] << 16)).reshape(krot, K // 2).contiguous()
        self.scales = None if channel_scales is None else channel_scales.float().reshape(-1).contiguous()
        self.krot, self.K = krot, K

    def to(self, device, dtype=None):
        """A copy on `device` (the angles and scales stay fp32)."""
        out = object.__new__(PairwiseRotation)
        out.krot, out.K = self.krot, self.K
        for n in ("cos", "sin", "pairs", "scales"):
            t = getattr(self, n)
            setattr(out, n, None if t is None else t.to(device))
        return out

    def rotate_ref(self, x: torch.Tensor) -> torch.Tensor:
        """fp32 re-statement: scale, then each round's pair rotations."""
        T, K = x.shape
        t = x.float() * (self.scales[None] if self.scales is not None else 1.0)
        t = t.reshape(T, K // GROUP, GROUP).clone()
        cos, sin, pr = self.cos.cpu(), self.sin.cpu(), self.pairs.cpu()
        for k in range(self.krot):
            c = cos[k].reshape(K // GROUP, GROUP // 2).to(t.device)
            s = sin[k].reshape(K // GROUP, GROUP // 2).to(t.device)
            p = pr[k].reshape(K // GROUP, GROUP // 2)
            i, j = (p & 0xFFFF).long().to(t.device), (p >> 16).long().to(t.device)
            a = torch.gather(t, 2, i[None].expand(T, -1, -1))
            b = torch.gather(t, 2, j[None].expand(T, -1, -1))
            t.scatter_(2, i[None].expand(T, -1, -1), a * c + b * s)
            t.scatter_(2, j[None].expand(T, -1, -1), b * c - a * s)
        return t.reshape(T, K).to(x.dtype)

    def rotate(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            return self.rotate_ref(x)
        T, K = x.shape
        x = x.contiguous()
        out = torch.empty_like(x)
        _lib.check(_lib.lib().b200_pair_rotate(x.data_ptr(), x.stride(0), T, K, self.cos.data_ptr(),
                                               self.sin.data_ptr(), self.pairs.data_ptr(), _lib.ptr(self.scales),
                                               self.krot, out.data_ptr(), out.stride(0),
                                               _lib.stream_ptr(x.device)), "pair_rotate")
        _lib.count(1)
        return out


class HadamardTransform:
    """Block Walsh-Hadamard transform with sign flips (Prism Hadamard
    checkpoints): forward y = H_b(s * x) / sqrt(b) per block of b channels;
    H_b is orthogonal after the scaling, so the inverse is s * H_b(y) / sqrt(b)."""

    def __init__(self, block: int, signs: torch.Tensor | None = None):
        assert block >= 2 and block & (block - 1) == 0
        self.block = block
        self.signs = None if signs is None else signs.float().reshape(-1).contiguous()

    def to(self, device, dtype=None):
        return HadamardTransform(self.block, None if self.signs is None else self.signs.to(device))

    def _ref(self, x, inverse):
        T, K = x.shape
        b = self.block
        t = x.to(torch.promote_types(x.dtype, torch.float32))
        if self.signs is not None and not inverse:
            t = t * self.signs.to(t.device)
        t = t.reshape(T, K // b, b)
        h = 1
        while h < b:
            t = t.reshape(T, K // b, b // (2 * h), 2, h)
            a, c = t[..., 0, :], t[..., 1, :]
            t = torch.stack([a + c, a - c], -2)
            h *= 2
        t = t.reshape(T, K) / (b ** 0.5)
        if self.signs is not None and inverse:
            t = t * self.signs.to(t.device)
        return t.to(x.dtype)

    def _apply(self, x, inverse):
        if not x.is_cuda:
            return self._ref(x, inverse)
        T, K = x.shape
        x = x.contiguous()
        out = torch.empty_like(x)
        _lib.check(_lib.lib().b200_block_hadamard(x.data_ptr(), x.stride(0), T, K, self.block, _lib.ptr(self.signs),
                                                  1 if inverse else 0, out.data_ptr(), out.stride(0),
                                                  _lib.stream_ptr(x.device)), "block_hadamard")
        _lib.count(1)
        return out

    def rotate(self, x):
        return self._apply(x, False)

    def inverse(self, y):
        return self._apply(y, True)


class RotatedWeight:
    """Output-row blocks [(rotation or None, weight [N_i, K])] of one
    projection; `glu` marks a gate/up pair (two blocks) whose outputs are
    combined by the GLU activation instead of concatenated."""

    def __init__(self, parts: list, glu: bool = False):
        self.parts = parts
        self.glu = glu
        self.shape = (sum(w.shape[0] for _, w in parts), parts[0][1].shape[1])

    def to(self, device=None, dtype=None):
        out = []
        for r, w in self.parts:
            out.append((r.to(device) if r is not None else None,
                        w.to(device) if not isinstance(w, torch.Tensor) else w.to(device=device, dtype=dtype or w.dtype)))
        return RotatedWeight(out, self.glu)

    def tensors(self):
        for i, (r, w) in enumerate(self.parts):
            if isinstance(w, torch.Tensor):
                yield f"{i}", w

    def gemm(self, x: torch.Tensor, epi: str = "none", bias=None, residual=None, out=None):
        from .linear import _GLU, gemm

        rotated = {}

        def rx(r):
            if r is None:
                return x
            key = id(r)
            if key not in rotated:
                rotated[key] = r.rotate(x)
            return rotated[key]

        if self.glu:
            assert epi in _GLU and len(self.parts) == 2, "a rotated gate/up pair needs a GLU epilogue"
            (rg, wg), (ru, wu) = self.parts
            g = gemm(rx(rg), wg, epi="f32")
            u = gemm(rx(ru), wu, epi="f32")
            if bias is not None:  # bias is interleaved like the fused layout; not produced by ParoQuant
                raise NotImplementedError("biased rotated gate/up")
            from .reference import glu_act_ref

            y = glu_act_ref(epi, g.to(x.dtype).float(), u.to(x.dtype).float()).to(x.dtype)
            if out is not None:
                out.copy_(y)
                return out
            return y
        ys, o = [], 0
        for r, w in self.parts:
            n = w.shape[0]
            b = None if bias is None else bias[o:o + n]
            ys.append(gemm(rx(r), w, epi="f32" if epi == "f32" else "none", bias=b))
            o += n
        y = torch.cat(ys, -1) if len(ys) > 1 else ys[0]
        if epi == "add":
            y = (y.float() + residual.float()).to(x.dtype)
        elif epi not in ("none", "f32"):
            raise NotImplementedError(f"epilogue {epi} on a rotated weight")
        if out is not None:
            out.copy_(y)
            return out
        return y


def awq_unpack(packed: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """AutoAWQ int32 words [R, C/8] -> codes [R, C] (undoing AutoAWQ's
    [0, 2, 4, 6, 1, 3, 5, 7] nibble order)."""
    R, W = packed.shape
    shifts = torch.arange(8, dtype=torch.int64) * bits
    raw = (packed.to(torch.int64)[..., None] >> shifts) & ((1 << bits) - 1)
    order = torch.tensor([0, 4, 1, 5, 2, 6, 3, 7])
    return raw[..., order].reshape(R, W * 8).to(torch.int32)


def awq_to_quantized(qweight, qzeros, scales, group_size: int):
    """AutoAWQ (qweight [K, N/8], qzeros [K/gs, N/8], scales [K/gs, N]) ->
    an affine :class:`QuantizedWeight` [N, K] (bias = -scale * zero)."""
    from .qlinear import QuantizedWeight

    q = awq_unpack(qweight).t().contiguous()  # [N, K]
    z = awq_unpack(qzeros).float()  # [K/gs, N]
    s = scales.float()
    return QuantizedWeight.from_codes(q, s.t(), (-s * z).t(), 4, group_size)
