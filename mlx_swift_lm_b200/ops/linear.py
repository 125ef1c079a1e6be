"""Dense GEMM entry points (tcgen05 kernel on CUDA, fp32 oracle on CPU)."""
from __future__ import annotations

import threading

import torch

from . import _lib
from .qlinear import QuantizedWeight
from .reference import gemm_ref

_EPI = {"none": 0, "swiglu": 1, "f32": 2, "add": 3, "geglu": 4, "swiglu_oai": 5, "gelu": 6, "gelu_tanh": 7, "quick_gelu": 8,
        "relu2": 9}
_GLU = ("swiglu", "geglu", "swiglu_oai")
_SMS: dict[int, int] = {}

# Row roles of the step being run: (T, nd) = the step's token count and how many
# leading rows are decode rows. GEMMs over exactly T rows then run the decode
# rows with the (N, K)-chosen split-K and the prefill rows with no split (one
# 128 x 256 tile per CTA over the whole K range). Each token's arithmetic depends
# only on its role, never on the batch, so batch-composition invariance holds,
# and prefill GEMMs are not chopped into 8 K-slices reduced over the cluster.
_ROLES = threading.local()


class row_roles:
    """Context: the current step has `T` tokens, the first `nd` of them decode rows."""

    def __init__(self, T: int, nd: int):
        self.v = (int(T), int(nd))

    def __enter__(self):
        self.prev = getattr(_ROLES, "v", None)
        _ROLES.v = self.v
        return self

    def __exit__(self, *exc):
        _ROLES.v = self.prev
        return False


def _split_rows(x: torch.Tensor):
    """(nd, T) when x holds the current step's rows and both roles are present,
    (0, T) for an all-prefill step, else None (default split rule)."""
    v = getattr(_ROLES, "v", None)
    if v is None or x.shape[0] != v[0] or v[1] >= v[0]:
        return None
    return v[1], v[0]


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _SMS.get(idx)
    if n is None:
        n = _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return n


def gemm(x: torch.Tensor, w: torch.Tensor, epi: str = "none", residual: torch.Tensor | None = None,
         out: torch.Tensor | None = None, bias: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """y = epi(x @ w.T + bias). x [M, K], w [N, K] (bf16 on CUDA).

    epi = "swiglu" / "geglu" / "swiglu_oai": w holds interleaved 64-row gate/up
    blocks ([2F, K]); y is [M, F].  epi = "f32": fp32 output.
    epi = "add": y = x @ w.T + residual.  `splits` overrides the split-K count.
    """
    if bias is not None and x.is_cuda and bias.dtype != x.dtype:  # the epilogues read biases in x's dtype
        bias = bias.to(x.dtype)
    if isinstance(w, QuantizedWeight):
        return gemm_q(x, w, epi, residual, out, bias, splits)
    if not isinstance(w, torch.Tensor) and hasattr(w, "gemm"):  # e.g. rotation.RotatedWeight
        return w.gemm(x, epi, bias=bias, residual=residual, out=out)
    if not x.is_cuda:
        y = gemm_ref(x, w, epi, residual, bias=bias)
        if out is not None:
            out.copy_(y)
            return out
        return y
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K, (x.shape, w.shape)
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16, (x.dtype, w.dtype)
    if x.stride(1) != 1:
        x = x.contiguous()
    n_out = N // 2 if epi in _GLU else N
    if out is None:
        out = torch.empty((M, n_out), dtype=torch.float32 if epi == "f32" else torch.bfloat16, device=x.device)
    roles = _split_rows(x) if splits == 0 else None
    if roles is not None:
        nd, T = roles
        r = residual
        if nd:
            gemm(x[:nd], w, epi, r[:nd] if r is not None else None, out[:nd], bias, 0)
        gemm(x[nd:], w, epi, r[nd:] if r is not None else None, out[nd:], bias, 1)
        return out
    rc = _lib.lib().b200_gemm_bf16(x.data_ptr(), M, K, x.stride(0), w.data_ptr(), N, w.stride(0), out.data_ptr(),
                                   out.stride(0), _lib.ptr(residual),
                                   residual.stride(0) if residual is not None else 0, _lib.ptr(bias), _EPI[epi],
                                   num_sms(x.device), int(splits), _lib.stream_ptr(x.device))
    _lib.check(rc, f"gemm M={M} N={N} K={K} epi={epi}")
    _lib.count(1)
    return out


def gemm_q(x: torch.Tensor, w: QuantizedWeight, epi: str = "none", residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None, bias: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """:func:`gemm` with an affine-quantised weight (dequantised tile by tile
    in shared memory by the tcgen05 kernel; CPU: the fp32 oracle over the
    dequantised weight)."""
    if not x.is_cuda:
        y = gemm_ref(x, w.dequantize(torch.float32).to(x.dtype), epi, residual, bias=bias)
        if out is not None:
            out.copy_(y)
            return out
        return y
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K, (x.shape, w.shape)
    assert x.dtype == torch.bfloat16 and w.scales_t.dtype == torch.bfloat16
    if x.stride(1) != 1:
        x = x.contiguous()
    n_out = N // 2 if epi in _GLU else N
    if out is None:
        out = torch.empty((M, n_out), dtype=torch.float32 if epi == "f32" else torch.bfloat16, device=x.device)
    roles = _split_rows(x) if splits == 0 else None
    if roles is not None:
        nd, T = roles
        r = residual
        if nd:
            gemm_q(x[:nd], w, epi, r[:nd] if r is not None else None, out[:nd], bias, 0)
        gemm_q(x[nd:], w, epi, r[nd:] if r is not None else None, out[nd:], bias, 1)
        return out
    rc = _lib.lib().b200_gemm_q(x.data_ptr(), M, K, x.stride(0), w.tiled().data_ptr(), N, w.kernel_bits, w.gs,
                                out.data_ptr(), out.stride(0),
                                _lib.ptr(residual), residual.stride(0) if residual is not None else 0,
                                _lib.ptr(bias), _EPI[epi], num_sms(x.device), int(splits),
                                _lib.stream_ptr(x.device))
    _lib.check(rc, f"gemm_q M={M} N={N} K={K} bits={w.bits} gs={w.gs} epi={epi}")
    _lib.count(1)
    return out


class _NoWorkspace:
    """The cluster split-K GEMM needs no global workspace; kept so callers that
    reserve memory before CUDA-graph capture have nothing to do."""

    def reserve(self, device, nbytes):
        return None


WORKSPACE = _NoWorkspace()


def gemm_qkv_rope(x: torch.Tensor, w: torch.Tensor, bias, positions, slots, cos_sin, q_norm, k_norm, eps: float,
                  k_cache, v_cache, H: int, KVH: int, k_scale=None, v_scale=None, q_out=None,
                  splits: int = 0) -> torch.Tensor:
    """q|k|v projection with qk-norm + RoPE + paged K/V append in the GEMM
    epilogue (head dim 128, full non-interleaved rotary): returns q [M, H, 128]
    and writes the tokens' K/V into the cache at `slots`. Same result as
    ``gemm`` followed by ``qk_norm_rope_kv``, without the projection's round
    trip through memory and without the separate launch."""
    M, K = x.shape
    N = w.shape[0]
    assert N == (H + 2 * KVH) * 128 and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    if x.stride(1) != 1:
        x = x.contiguous()
    if bias is not None and bias.dtype != x.dtype:
        bias = bias.to(x.dtype)
    if q_out is None:
        q_out = torch.empty((M, H, 128), dtype=torch.bfloat16, device=x.device)
    fp8 = k_cache is not None and k_cache.dtype == torch.float8_e4m3fn
    num_slots = k_cache.shape[0] * 16 if k_cache is not None else 0
    roles = _split_rows(x) if splits == 0 else None
    if roles is not None:
        nd, T = roles
        parts = ((0, nd, 0), (nd, T, 1)) if nd else ((0, T, 1),)
    else:
        parts = ((0, M, splits),)
    for lo, hi, sp in parts:
        rc = _lib.lib().b200_gemm_qkv_rope(
            x[lo:hi].data_ptr(), hi - lo, K, x.stride(0), w.data_ptr(), N, w.stride(0), _lib.ptr(bias),
            positions[lo:hi].data_ptr(), _lib.ptr(slots[lo:hi] if slots is not None else None), cos_sin.data_ptr(),
            _lib.ptr(q_norm), _lib.ptr(k_norm), float(eps), q_out[lo:hi].data_ptr(), _lib.ptr(k_cache),
            _lib.ptr(v_cache), 1 if fp8 else 0, _lib.ptr(k_scale), _lib.ptr(v_scale), H, KVH, num_slots,
            num_sms(x.device), sp, _lib.stream_ptr(x.device))
        _lib.check(rc, f"gemm_qkv_rope M={hi - lo} N={N} K={K}")
        _lib.count(1)
    return q_out
