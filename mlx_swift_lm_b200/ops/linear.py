"""Dense GEMM entry points (tcgen05 kernel on CUDA, fp32 oracle on CPU)."""
from __future__ import annotations

import torch

from . import _lib
from .qlinear import QuantizedWeight
from .reference import gemm_ref

_EPI = {"none": 0, "swiglu": 1, "f32": 2, "add": 3, "geglu": 4, "swiglu_oai": 5, "gelu": 6, "gelu_tanh": 7, "quick_gelu": 8,
        "relu2": 9}
_GLU = ("swiglu", "geglu", "swiglu_oai")
_SMS: dict[int, int] = {}


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
