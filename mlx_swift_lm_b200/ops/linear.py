"""Dense GEMM entry points (tcgen05 kernel on CUDA, fp32 oracle on CPU)."""
from __future__ import annotations

import threading

import torch

from . import _lib
from .reference import gemm_ref

_EPI = {"none": 0, "swiglu": 1, "f32": 2, "add": 3, "geglu": 4, "swiglu_oai": 5}
_GLU = ("swiglu", "geglu", "swiglu_oai")


class _Workspace:
    """Per-device split-K workspace and self-resetting tile counters.

    Ops on one device share it; every op in this framework runs its GEMMs on
    one stream at a time (the engine stream, or the stream a CUDA graph was
    captured on), so uses never overlap."""

    def __init__(self):
        self.lock = threading.Lock()
        self.ws: dict[int, torch.Tensor] = {}
        self.ctr: dict[int, torch.Tensor] = {}
        self.sms: dict[int, int] = {}

    def get(self, device: torch.device, ws_bytes: int, n_ctr: int):
        idx = device.index if device.index is not None else torch.cuda.current_device()
        with self.lock:
            ws = self.ws.get(idx)
            if ws is None or ws.numel() * 4 < ws_bytes:
                size = max(ws_bytes, 64 << 20)
                ws = torch.empty(size // 4, dtype=torch.float32, device=device)
                self.ws[idx] = ws
            ctr = self.ctr.get(idx)
            if ctr is None or ctr.numel() < n_ctr:
                ctr = torch.zeros(max(n_ctr, 1 << 16), dtype=torch.int32, device=device)
                self.ctr[idx] = ctr
            if idx not in self.sms:
                self.sms[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
            return ws, ctr, self.sms[idx]

    def reserve(self, device: torch.device, ws_bytes: int):
        """Grow the workspace ahead of CUDA-graph capture."""
        self.get(device, ws_bytes, 1 << 16)


WORKSPACE = _Workspace()


def gemm(x: torch.Tensor, w: torch.Tensor, epi: str = "none", residual: torch.Tensor | None = None,
         out: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """y = epi(x @ w.T). x [M, K], w [N, K] (bf16 on CUDA).

    epi = "swiglu": w holds interleaved 64-row gate/up blocks ([2F, K]); y is [M, F].
    epi = "f32": fp32 output.  epi = "add": y = x @ w.T + residual.
    """
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
    L = _lib.lib()
    sms = WORKSPACE.sms.get(x.device.index)
    if sms is None:
        WORKSPACE.get(x.device, 0, 1)
        sms = WORKSPACE.sms[x.device.index]
    ws_bytes = L.b200_gemm_workspace_bytes(M, N, K, sms)
    ws, ctr, _ = WORKSPACE.get(x.device, ws_bytes, 1 << 16)
    rc = L.b200_gemm_bf16(x.data_ptr(), M, K, x.stride(0), w.data_ptr(), N, w.stride(0), out.data_ptr(),
                          out.stride(0), _lib.ptr(residual), residual.stride(0) if residual is not None else 0,
                          _lib.ptr(bias), _EPI[epi], ws.data_ptr(), ws.numel() * 4, ctr.data_ptr(), ctr.numel(), sms, 0,
                          _lib.stream_ptr(x.device))
    _lib.check(rc, f"gemm M={M} N={N} K={K} epi={epi}")
    _lib.count(1)
    return out
