"""RMSNorm / residual / RoPE / KV-append / embedding ops."""
from __future__ import annotations

import torch

from . import _lib
from . import reference as ref


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor | None, w: torch.Tensor, eps: float,
                out: torch.Tensor | None = None, offset_one: bool = False) -> torch.Tensor:
    """x <- x + delta (in place, rounded to x.dtype); returns RMSNorm(x) * w."""
    if not x.is_cuda:
        r, y = ref.add_rmsnorm_ref(x, delta, w, eps, offset_one)
        if delta is not None:
            x.copy_(r)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, H = x.shape
    if out is None:
        out = torch.empty_like(x)
    rc = _lib.lib().b200_add_rmsnorm(x.data_ptr(), _lib.ptr(delta), w.data_ptr(), out.data_ptr(), T, H,
                                     x.stride(0), delta.stride(0) if delta is not None else 0, out.stride(0),
                                     float(eps), 1 if offset_one else 0, _lib.stream_ptr(x.device))
    _lib.check(rc, "add_rmsnorm")
    _lib.count(1)
    return out


def add_layernorm(x: torch.Tensor, delta: torch.Tensor | None, w: torch.Tensor, b: torch.Tensor | None, eps: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """x <- x + delta (in place, rounded to x.dtype); returns LayerNorm(x) * w + b
    (`out` may be x itself: the post-norm residual of BERT-family encoders)."""
    if not x.is_cuda:
        if delta is not None:
            x.copy_((x.float() + delta.float()).to(x.dtype))
        y = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), w.float(),
                                           None if b is None else b.float(), eps).to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, H = x.shape
    if out is None:
        out = torch.empty_like(x)
    rc = _lib.lib().b200_add_layernorm(x.data_ptr(), _lib.ptr(delta), w.data_ptr(), _lib.ptr(b), out.data_ptr(), T, H,
                                       x.stride(0), delta.stride(0) if delta is not None else 0, out.stride(0),
                                       float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "add_layernorm")
    _lib.count(1)
    return out


def rmsnorm(x, w, eps, offset_one=False):
    return add_rmsnorm(x, None, w, eps, offset_one=offset_one)


def qk_norm_rope_kv(qkv: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor | None, cos_sin: torch.Tensor,
                    rot_dim: int, interleaved: bool, q_norm: torch.Tensor | None, k_norm: torch.Tensor | None,
                    eps: float, k_cache: torch.Tensor | None, v_cache: torch.Tensor | None, H: int, KVH: int, D: int,
                    k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
                    q_out: torch.Tensor | None = None, return_kv: bool = False):
    """Split fused qkv [T, (H+2KVH)*D], qk-norm, RoPE, and append K/V to the
    paged cache at `slots` (page*16+offset; -1 skips). Returns q [T, H, D]
    (and k, v [T, KVH, D] when return_kv)."""
    T = qkv.shape[0]
    if not qkv.is_cuda:
        q, k, v = ref.qk_norm_rope_kv_ref(qkv, positions, slots, cos_sin, rot_dim, interleaved, q_norm, k_norm, eps,
                                          k_cache, v_cache, H, KVH, D, k_scale, v_scale)
        if q_out is not None:
            q_out.copy_(q)
            q = q_out
        return (q, k, v) if return_kv else q
    if q_out is None:
        q_out = torch.empty((T, H, D), dtype=qkv.dtype, device=qkv.device)
    k_out = v_out = None
    if return_kv:
        k_out = torch.empty((T, KVH, D), dtype=qkv.dtype, device=qkv.device)
        v_out = torch.empty((T, KVH, D), dtype=qkv.dtype, device=qkv.device)
    kv_fp8 = k_cache is not None and k_cache.dtype == torch.float8_e4m3fn
    num_slots = k_cache.shape[0] * 16 if k_cache is not None else 0
    rc = _lib.lib().b200_qk_norm_rope_kv(
        qkv.data_ptr(), T, qkv.stride(0), positions.data_ptr(), _lib.ptr(slots), cos_sin.data_ptr(), rot_dim,
        1 if interleaved else 0, _lib.ptr(q_norm), _lib.ptr(k_norm), float(eps), q_out.data_ptr(),
        _lib.ptr(k_cache), _lib.ptr(v_cache), 1 if kv_fp8 else 0, _lib.ptr(k_scale), _lib.ptr(v_scale), H, KVH, D,
        num_slots, _lib.ptr(k_out), _lib.ptr(v_out), _lib.stream_ptr(qkv.device))
    _lib.check(rc, "qk_norm_rope_kv")
    _lib.count(1)
    return (q_out, k_out, v_out) if return_kv else q_out


def embedding(ids: torch.Tensor, table: torch.Tensor, scale: float = 1.0, out: torch.Tensor | None = None):
    if not ids.is_cuda:
        y = table[ids.long()]
        if scale != 1.0:
            y = (y.float() * scale).to(table.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T = ids.shape[0]
    H = table.shape[1]
    if out is None:
        out = torch.empty((T, H), dtype=table.dtype, device=table.device)
    rc = _lib.lib().b200_embedding(ids.data_ptr(), table.data_ptr(), out.data_ptr(), T, H, table.shape[0],
                                   float(scale), _lib.stream_ptr(ids.device))
    _lib.check(rc, "embedding")
    _lib.count(1)
    return out


def silu_mul(gu: torch.Tensor, out: torch.Tensor | None = None):
    """[T, 2F] laid out [gate | up] -> silu(gate) * up."""
    T, F2 = gu.shape
    F = F2 // 2
    if not gu.is_cuda:
        y = (torch.nn.functional.silu(gu[:, :F].float()) * gu[:, F:].float()).to(gu.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty((T, F), dtype=gu.dtype, device=gu.device)
    rc = _lib.lib().b200_silu_mul(gu.data_ptr(), out.data_ptr(), T, F, gu.stride(0), out.stride(0),
                                  _lib.stream_ptr(gu.device))
    _lib.check(rc, "silu_mul")
    _lib.count(1)
    return out


def xielu(x: torch.Tensor, params: torch.Tensor) -> torch.Tensor:
    """xIELU activation in place (Apertus MLPs). params = raw (alpha_p,
    alpha_n, beta, eps) of the layer (fp32 [4]); see xielu_ref."""
    if not x.is_cuda:
        x.copy_(ref.xielu_ref(x, params))
        return x
    assert x.dtype == torch.bfloat16 and x.is_contiguous()
    rc = _lib.lib().b200_xielu(x.data_ptr(), x.numel(), params.data_ptr(), _lib.stream_ptr(x.device))
    _lib.check(rc, "xielu")
    _lib.count(1)
    return x


_lib.register_signatures({"b200_xielu": (_lib.i32, [_lib.vp, _lib.i64, _lib.vp, _lib.vp])})
