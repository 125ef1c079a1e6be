"""MoE routing and expert computation: router top-k, sort tokens by expert,
per-expert GLU MLP, weighted un-sort. Parity: MLXLMCommon/MoERouterTopK.swift:22
(router top-k, ties to the lower expert id) and the SwitchGLU of
MLXLMCommon/SwitchLayers.swift:478 (gatherSort :244, scatterUnsort :257,
weightedExpertUnsort :149).

On CUDA every step runs on the kernels of ``csrc/kernels/moe.cu`` with no host
synchronisation (so the MoE layer captures into the decode CUDA graph):

    route_topk   warp-per-token softmax/top-k
    sort         stable counting sort of the T*k (token, expert) pairs plus a
                 device work list of (expert, first row, rows <= BN) chunks
    gather       activation rows in expert order
    grouped GEMM tcgen05 tiles over (weight tile, chunk); the gate/up GEMM
                 applies the GLU in its epilogue, the down GEMM adds the bias
    combine      out[t] = sum_j w[t, j] * y[pos(t, j)] in slot order j

CPU tensors take the plain PyTorch path (used by the CPU test suite).
"""
from __future__ import annotations

import os

import torch

from . import _lib
from .linear import gemm
from .qlinear import QuantizedWeight

_EPI = {"none": 0, "swiglu": 1, "geglu": 4, "swiglu_oai": 5}

_lib.register_signatures({
    "b200_moe_route_topk": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.vp,
                                       _lib.vp, _lib.i32, _lib.i32, _lib.f32, _lib.vp]),
    "b200_moe_sort": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.vp, _lib.vp, _lib.vp,
                                 _lib.vp, _lib.vp]),
    "b200_moe_gather": (_lib.i32, [_lib.vp, _lib.i32, _lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.vp]),
    "b200_moe_combine": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.vp, _lib.i32, _lib.vp, _lib.vp,
                                    _lib.vp, _lib.vp]),
    "b200_moe_grouped_gemm": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.i32, _lib.vp,
                                         _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.vp, _lib.i32, _lib.i32,
                                         _lib.vp]),
    "b200_moe_grouped_gemm_q": (_lib.i32, [_lib.vp, _lib.i32, _lib.i32, _lib.vp, _lib.i32, _lib.i32, _lib.i32,
                                           _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.i32, _lib.vp, _lib.vp,
                                           _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.vp]),
}, status_tags=("moe",))


_MODES = {"softmax_topk": 0, "topk_softmax": 1, "sigmoid_group": 2}


def route_topk(logits: torch.Tensor, k: int, mode: str = "softmax_topk", norm_topk: bool = True,
               bias: torch.Tensor | None = None, n_group: int = 1, topk_group: int = 1, scale: float = 1.0):
    """Router top-k over fp32 logits [T, E]. softmax_topk: softmax over experts
    then top-k (optionally renormalised); topk_softmax: top-k logits then
    softmax over the k (softmax_topk and sigmoid_group weights are multiplied
    by `scale`); sigmoid_group: sigmoid scores, selection by score +
    `bias` inside the `topk_group` best of `n_group` groups (group score =
    sum of its two best biased scores), weights = the chosen sigmoid scores
    (renormalised when `norm_topk` and k > 1) times `scale`. Returns
    (weights [T, k] fp32, ids [T, k] int32 on CUDA, int64 on CPU)."""
    T, E = logits.shape
    if logits.is_cuda:
        assert E <= 256 and k <= 16, "router kernel supports up to 256 experts and k <= 16"
        lg = logits.float().contiguous()
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        b = None if bias is None else bias.float().contiguous()
        _lib.check(_lib.lib().b200_moe_route_topk(lg.data_ptr(), T, E, k, _MODES[mode], 1 if norm_topk else 0,
                                                  ids.data_ptr(), w.data_ptr(), _lib.ptr(b), int(n_group),
                                                  int(topk_group), float(scale), _lib.stream_ptr(logits.device)),
                   "moe_route_topk")
        _lib.count(1)
        return w, ids
    if mode == "topk_softmax":
        v, idx = torch.topk(logits.float(), k, dim=-1)
        return torch.softmax(v, dim=-1), idx
    if mode == "sigmoid_group":
        return _route_sigmoid_group_ref(logits.float(), k, norm_topk, bias, n_group, topk_group, scale)
    p = torch.softmax(logits.float(), dim=-1)
    if n_group > 1:  # group-limited greedy: groups ranked by their best probability
        g = p.reshape(T, n_group, E // n_group)
        keep = _stable_topk(g.max(-1).values, topk_group)
        mask = torch.zeros(T, n_group, dtype=torch.bool, device=p.device)
        mask.scatter_(1, keep, True)
        p = torch.where(mask[..., None], g, torch.zeros_like(g)).reshape(T, E)
    idx = _stable_topk(p, k)
    w = torch.gather(p, 1, idx)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True)
    return w * scale, idx


def _stable_topk(x: torch.Tensor, k: int):
    """Top-k along the last dim with ties to the lower index."""
    n = x.shape[-1]
    key = x.double() - torch.arange(n, dtype=torch.float64, device=x.device) * 1e-12
    return torch.topk(key, k, dim=-1).indices


def _route_sigmoid_group_ref(lg, k, norm_topk, bias, n_group, topk_group, scale):
    T, E = lg.shape
    s = torch.sigmoid(lg)
    sel = s + (bias.float() if bias is not None else 0.0)
    if n_group > 1:
        g = sel.reshape(T, n_group, E // n_group)
        top2 = torch.sort(g, dim=-1, descending=True).values[..., :2].sum(-1) if E // n_group > 1 else g[..., 0]
        keep = _stable_topk(top2, topk_group)
        mask = torch.zeros(T, n_group, dtype=torch.bool, device=lg.device)
        mask.scatter_(1, keep, True)
        sel = torch.where(mask[..., None], g, torch.zeros_like(g)).reshape(T, E)
    idx = _stable_topk(sel, k)
    w = torch.gather(s, 1, idx)
    if norm_topk and k > 1:
        w = w / w.sum(-1, keepdim=True)
    return w * scale, idx


def chunk_rows(P: int, E: int) -> int:
    """Row cap of one grouped-GEMM chunk: the smallest tile width that holds the
    average rows per expert (a function of the shape only, so it is fixed per
    captured graph)."""
    avg = (P + E - 1) // max(E, 1)
    for bn in (16, 32, 64):
        if avg <= bn:
            return bn
    return 128


# quantised experts, chunks of <= 32 rows (decode): B200LM_MOE_PERSISTENT=1 runs
# persistent CTAs (one per SM, looping over (chunk, weight tile) items). Off by
# default: with one CTA per SM it has half the dequantising warps per SM of the
# two-CTAs-per-SM launch, and the dequantisation is the limit at decode sizes.
PERSISTENT = [os.environ.get("B200LM_MOE_PERSISTENT", "0") == "1"]
# MXFP4 experts: f16 operands (hardware e2m1 pair conversion, f16 activations
# and gate/up rows) when every block scale keeps the weights normal f16
F16_MXFP4 = [os.environ.get("B200LM_MOE_F16", "1") != "0"]


def _f16_path(W) -> bool:
    return (F16_MXFP4[0] and isinstance(W, QuantizedWeight) and W.kernel_bits == -4 and W.gs == 32
            and W.f16_scales_ok())


def _grouped(L, xs, P, K, W, E, N, Y, ldy, bias, epi, chunks, n_chunks, max_chunks, BN, st, what, f16=False,
             y_f16=False):
    if isinstance(W, QuantizedWeight):
        from .linear import num_sms

        rec = W.tiled_natural() if f16 else W.tiled()
        rc = L.b200_moe_grouped_gemm_q(xs.data_ptr(), P, K, rec.data_ptr(), W.kernel_bits, W.gs, E, N, Y.data_ptr(),
                                       ldy, _lib.ptr(bias), epi, chunks.data_ptr(), n_chunks.data_ptr(), max_chunks,
                                       BN, num_sms(xs.device) if PERSISTENT[0] else 0, 1 if f16 else 0,
                                       1 if y_f16 else 0, st)
    else:
        rc = L.b200_moe_grouped_gemm(xs.data_ptr(), P, K, W.data_ptr(), E, N, Y.data_ptr(), ldy, _lib.ptr(bias), epi,
                                     chunks.data_ptr(), n_chunks.data_ptr(), max_chunks, BN, st)
    _lib.check(rc, f"moe_grouped_gemm {what}")


def _moe_experts_cuda(h, experts_gu, experts_d, w, idx, epi, gu_bias, d_bias, rot_in=None, rot_mid=None):
    if rot_in is not None:
        h = rot_in.rotate(h)
    T, K = h.shape
    k = idx.shape[1]
    if isinstance(experts_gu, QuantizedWeight):
        E = experts_gu.num_experts
        N2 = experts_gu.shape[0] // E
        F = experts_d.shape[1]
    else:
        E, N2, _ = experts_gu.shape
        F = experts_d.shape[2]
    assert N2 == 2 * F and N2 % 128 == 0, "gate/up rows must be 2*F, a multiple of 128 (64-row interleave)"
    P = T * k
    dev = h.device
    BN = chunk_rows(P, E)
    max_chunks = (P + BN - 1) // BN + E
    ids = idx.to(torch.int32).contiguous()
    w = w.float().contiguous()
    perm = torch.empty(P, dtype=torch.int32, device=dev)
    pos = torch.empty(P, dtype=torch.int32, device=dev)
    chunks = torch.empty(max_chunks * 3, dtype=torch.int32, device=dev)
    n_chunks = torch.empty(1, dtype=torch.int32, device=dev)
    f16 = rot_mid is None and _f16_path(experts_gu) and _f16_path(experts_d)
    xs = torch.empty(P, K, dtype=torch.float16 if f16 else h.dtype, device=dev)
    gu = torch.empty(P, F, dtype=torch.float16 if f16 else h.dtype, device=dev)
    ys = torch.empty(P, K, dtype=h.dtype, device=dev)
    out = torch.empty(T, K, dtype=h.dtype, device=dev)
    L = _lib.lib()
    st = _lib.stream_ptr(dev)
    hc = h.contiguous()
    _lib.check(L.b200_moe_sort(ids.data_ptr(), P, E, BN, max_chunks, perm.data_ptr(), pos.data_ptr(),
                               chunks.data_ptr(), n_chunks.data_ptr(), st), "moe_sort")
    _lib.check(L.b200_moe_gather(hc.data_ptr(), K, perm.data_ptr(), P, k, xs.data_ptr(), 1 if f16 else 0, st),
               "moe_gather")
    _grouped(L, xs, P, K, experts_gu, E, N2, gu, F, gu_bias, _EPI[epi], chunks, n_chunks, max_chunks, BN, st,
             "gate/up", f16=f16, y_f16=f16)
    if rot_mid is not None:
        gu = rot_mid.rotate(gu)
    _grouped(L, gu, P, F, experts_d, E, K, ys, K, d_bias, 0, chunks, n_chunks, max_chunks, BN, st, "down", f16=f16)
    _lib.check(L.b200_moe_combine(ys.data_ptr(), T, K, pos.data_ptr(), w.data_ptr(), k, out.data_ptr(), None, None,
                                  st), "moe_combine")
    _lib.count(5)
    return out


def moe_experts(h, experts_gu, experts_d, w, idx, epi="swiglu", gu_bias=None, d_bias=None, rot_in=None,
                rot_mid=None):
    """h [T, K]; experts_gu [E, 2F, K] (64-row interleaved gate/up); experts_d [E, K, F];
    w [T, k] fp32 weights; idx [T, k] expert ids. Returns [T, K] in h.dtype.
    `rot_in` / `rot_mid`: ParoQuant rotations of the gate/up and down inputs
    shared by all experts (ops.rotation.PairwiseRotation)."""
    if h.is_cuda:
        return _moe_experts_cuda(h, experts_gu, experts_d, w, idx, epi, gu_bias, d_bias, rot_in, rot_mid)
    if rot_in is not None:
        h = rot_in.rotate(h)
    if isinstance(experts_gu, QuantizedWeight):
        E = experts_gu.num_experts
        experts_gu = torch.stack([experts_gu.expert(e).dequantize(torch.float32) for e in range(E)]).to(h.dtype)
        experts_d = torch.stack([experts_d.expert(e).dequantize(torch.float32) for e in range(E)]).to(h.dtype)
    T, K = h.shape
    k = idx.shape[1]
    flat = idx.reshape(-1).long()
    order = torch.argsort(flat, stable=True)
    tok = order // k
    wsorted = w.reshape(-1)[order]
    counts = torch.bincount(flat, minlength=experts_gu.shape[0]).tolist()  # experts dim
    out = torch.zeros((T, K), dtype=torch.float32, device=h.device)
    start = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        rows = tok[start:start + c]
        x = h.index_select(0, rows).contiguous()
        gu = gemm(x, experts_gu[e], epi=epi, bias=None if gu_bias is None else gu_bias[e])
        if rot_mid is not None:
            gu = rot_mid.rotate(gu)
        y = gemm(gu, experts_d[e], bias=None if d_bias is None else d_bias[e])
        out.index_add_(0, rows, y.float() * wsorted[start:start + c, None])
        start += c
    return out.to(h.dtype)
