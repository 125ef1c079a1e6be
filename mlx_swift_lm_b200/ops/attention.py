"""Paged attention entry points: decode (split-KV) and prefill (chunked, causal)."""
from __future__ import annotations

import os
import threading

import torch

from . import _lib
from . import reference as ref

PART_TOKENS = ref.DECODE_PART_TOKENS
# bf16 pages use the tensor-core partition pass; set [0] = False for the CUDA-core kernel
USE_MMA_DECODE = [True]
# B200LM_FUSED_MERGE=1: the tensor-core decode merges its partitions in the last
# partition CTA of each row (one launch per layer). Off by default: measured on the
# Qwen3-8B 64-stream decode step it is 0.43 ms slower than the separate merge pass
# (the merging CTA's reads of the other partitions sit on the kernel's critical path).
USE_FUSED_MERGE = [os.environ.get("B200LM_FUSED_MERGE", "0") == "1"]


class _Scratch:
    """Per-device scratch for decode partials (grown on demand, reused)."""

    def __init__(self):
        self.lock = threading.Lock()
        self.bufs: dict[tuple, torch.Tensor] = {}

    def get(self, device, name, numel):
        key = (device.index, name)
        with self.lock:
            t = self.bufs.get(key)
            if t is None or t.numel() < numel:
                t = torch.empty(max(numel, 1 << 20), dtype=torch.float32, device=device)
                self.bufs[key] = t
            return t


SCRATCH = _Scratch()

_COUNTERS: dict[int, torch.Tensor] = {}


def merge_counters(device, n: int) -> torch.Tensor:
    """Per-device int32 arrival counters of the fused decode merge: zero
    between launches (each launch's merging CTAs reset theirs), allocated once
    at a fixed address so captured graphs keep using the same buffer. Launches
    that may overlap on the GPU (several streams) must not share them."""
    t = _COUNTERS.get(device.index)
    if t is None or t.numel() < n:
        t = torch.zeros(max(n, 1 << 16), dtype=torch.int32, device=device)
        _COUNTERS[device.index] = t
    return t


def decode_max_parts(max_seq_len: int) -> int:
    return max(1, (max_seq_len + PART_TOKENS - 1) // PART_TOKENS)


def paged_decode(q, k_cache, v_cache, page_table, seq_lens, scale, window=0, sinks=None, softcap=0.0,
                 k_scale=None, v_scale=None, max_parts=None, out=None):
    """q [B, H, D]; caches [P, KVH, 16, D]; page_table [B, maxp] int32; seq_lens [B] int32."""
    if not q.is_cuda:
        y = ref.paged_decode_ref(q, k_cache, v_cache, page_table, seq_lens, scale, window, sinks, softcap,
                                 k_scale, v_scale)
        if out is not None:
            out.copy_(y)
            return out
        return y
    B, H, D = q.shape
    KVH = k_cache.shape[1]
    if max_parts is None:
        max_parts = decode_max_parts(page_table.shape[1] * 16)
    if out is None:
        out = torch.empty_like(q)
    acc = SCRATCH.get(q.device, "dec_acc", B * H * max_parts * D)
    ml = SCRATCH.get(q.device, "dec_ml", B * H * max_parts * 2)
    kv_fp8 = k_cache.dtype == torch.float8_e4m3fn
    L = _lib.lib()
    if D == 512:  # wide heads: lanes split the head dim, then the common merge pass
        st = _lib.stream_ptr(q.device)
        rc = L.b200_paged_decode_wide_part(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), 1 if kv_fp8 else 0,
                                           _lib.ptr(k_scale), _lib.ptr(v_scale), page_table.data_ptr(),
                                           page_table.stride(0), seq_lens.data_ptr(), acc.data_ptr(), ml.data_ptr(),
                                           B, H, KVH, D, max_parts, int(window), float(scale), float(softcap),
                                           k_cache.shape[0], st)
        _lib.check(rc, "paged_decode_wide_part")
        rc = L.b200_paged_decode_merge(acc.data_ptr(), ml.data_ptr(), seq_lens.data_ptr(), _lib.ptr(sinks),
                                       out.data_ptr(), B, H, D, max_parts, int(window), st)
        _lib.check(rc, "paged_decode_merge")
        _lib.count(2)
        return out
    if not kv_fp8 and D in (64, 128, 256) and H // KVH <= (16 if D < 256 else 8) and USE_MMA_DECODE[0]:
        st = _lib.stream_ptr(q.device)
        if not USE_FUSED_MERGE[0]:
            rc = L.b200_paged_decode_mma_part(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                              page_table.data_ptr(), page_table.stride(0), seq_lens.data_ptr(),
                                              acc.data_ptr(), ml.data_ptr(), B, H, KVH, D, max_parts, int(window),
                                              float(scale), float(softcap), k_cache.shape[0], st)
            _lib.check(rc, "paged_decode_mma_part")
            rc = L.b200_paged_decode_merge(acc.data_ptr(), ml.data_ptr(), seq_lens.data_ptr(), _lib.ptr(sinks),
                                           out.data_ptr(), B, H, D, max_parts, int(window), st)
            _lib.check(rc, "paged_decode_merge")
            _lib.count(2)
            return out
        # partitions + merge in one launch (the last partition CTA of a row merges)
        cnt = merge_counters(q.device, B * KVH)
        rc = L.b200_paged_decode_mma(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), page_table.data_ptr(),
                                     page_table.stride(0), seq_lens.data_ptr(), acc.data_ptr(), ml.data_ptr(),
                                     cnt.data_ptr(), _lib.ptr(sinks), out.data_ptr(), B, H, KVH, D, max_parts,
                                     int(window), float(scale), float(softcap), k_cache.shape[0], st)
        _lib.check(rc, "paged_decode_mma")
        _lib.count(1)
        return out
    rc = L.b200_paged_decode(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), 1 if kv_fp8 else 0, _lib.ptr(k_scale),
        _lib.ptr(v_scale), page_table.data_ptr(), page_table.stride(0), seq_lens.data_ptr(), _lib.ptr(sinks),
        out.data_ptr(), acc.data_ptr(), ml.data_ptr(), B, H, KVH, D, max_parts, int(window), float(scale),
        float(softcap), k_cache.shape[0], _lib.stream_ptr(q.device))
    _lib.check(rc, "paged_decode")
    _lib.count(2)
    return out


USE_MMA_PREFILL = [True]  # tests flip it to cover the CUDA-core kernel


def prefill_tiles_mma(cu_q: list[int], qt: int = 64) -> list[tuple[int, int]]:
    """(row, query offset) work items of the tensor-core prefill kernel, the
    tiles that see the most keys (last offsets of long rows) first."""
    tiles = []
    for r in range(len(cu_q) - 1):
        n = cu_q[r + 1] - cu_q[r]
        for off in range(0, n, qt):
            tiles.append((r, off))
    tiles.sort(key=lambda t: -t[1])
    return tiles


def prefill_tiles(cu_q: list[int], G: int) -> list[tuple[int, int]]:
    qt = 128 // G
    tiles = []
    for r in range(len(cu_q) - 1):
        n = cu_q[r + 1] - cu_q[r]
        for off in range(0, n, qt):
            tiles.append((r, off))
    return tiles


def paged_prefill(q, k_cache, v_cache, page_table, cu_q, q_pos0, scale, window=0, sinks=None, softcap=0.0,
                  k_scale=None, v_scale=None, cu_q_host=None, out=None):
    """q [T, H, D] for rows' chunks; cu_q [R+1] int32; q_pos0 [R] int32 (first position of each chunk).
    window > 0: sliding window; 0: causal; < 0: bidirectional over each row's
    keys (encoders; bf16 pages, tensor-core kernel only)."""
    if not q.is_cuda:
        y = ref.paged_prefill_ref(q, k_cache, v_cache, page_table, cu_q, q_pos0, scale, window, sinks, softcap,
                                  k_scale, v_scale)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, H, D = q.shape
    KVH = k_cache.shape[1]
    G = H // KVH
    if out is None:
        out = torch.empty_like(q)
    if cu_q_host is None:
        cu_q_host = cu_q.tolist()
    if D == 512:
        if window < 0:
            raise ValueError("bidirectional attention is not served at head dim 512")
        return _prefill_wide(q, k_cache, v_cache, page_table, cu_q_host, q_pos0, scale, window, sinks, softcap,
                             k_scale, v_scale, out)
    if USE_MMA_PREFILL[0] and k_scale is None and k_cache.dtype == torch.bfloat16 and D in (64, 128, 256):
        # tensor-core kernel: 64-query tiles of one head, longest rows first
        tiles = prefill_tiles_mma(cu_q_host)
        tiles_t = torch.tensor(tiles, dtype=torch.int32).pin_memory().to(q.device, non_blocking=True)
        rc = _lib.lib().b200_paged_prefill_mma(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), page_table.data_ptr(), page_table.stride(0),
            cu_q.data_ptr(), q_pos0.data_ptr(), tiles_t.data_ptr(), len(tiles), _lib.ptr(sinks), out.data_ptr(), H,
            KVH, D, int(window), float(scale), float(softcap), k_cache.shape[0], _lib.stream_ptr(q.device))
        _lib.check(rc, "paged_prefill_mma")
        _lib.count(1)
        return out
    if window < 0:
        raise ValueError("bidirectional attention needs bf16 K/V pages and head_dim 64, 128 or 256")
    tiles = prefill_tiles(cu_q_host, G)
    tiles_t = torch.tensor(tiles, dtype=torch.int32).pin_memory().to(q.device, non_blocking=True)
    rc = _lib.lib().b200_paged_prefill_simt(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), page_table.data_ptr(), page_table.stride(0),
        cu_q.data_ptr(), q_pos0.data_ptr(), tiles_t.data_ptr(), len(tiles), _lib.ptr(sinks), out.data_ptr(), H, KVH,
        D, int(window), float(scale), float(softcap), k_cache.shape[0], _lib.stream_ptr(q.device))
    _lib.check(rc, "paged_prefill")
    _lib.count(1)
    return out


WIDE_PREFILL_SLICE = 128  # query tokens per partition pass (bounds the split-KV scratch)


def _prefill_wide(q, k_cache, v_cache, page_table, cu_q_host, q_pos0, scale, window, sinks, softcap, k_scale,
                  v_scale, out):
    """Prefill at head dim 512: every chunk token is a decode row of its own
    (its row's page table, context = its position + 1), attended by the wide
    decode kernel in slices of WIDE_PREFILL_SLICE tokens. The chunk's K/V are
    already in the pages, so each token sees exactly its causal (windowed)
    history, as the prefill kernels do."""
    T = q.shape[0]
    dev = q.device
    R = len(cu_q_host) - 1
    counts = torch.tensor([cu_q_host[r + 1] - cu_q_host[r] for r in range(R)], dtype=torch.int64)
    row = torch.repeat_interleave(torch.arange(R), counts).to(dev, non_blocking=True)
    start = torch.tensor(cu_q_host[:-1], dtype=torch.int64).to(dev, non_blocking=True)
    offs = torch.arange(T, device=dev, dtype=torch.int64) - start[row]
    seq_lens = (q_pos0.long()[row] + offs + 1).to(torch.int32)
    pt = page_table.index_select(0, row)
    max_parts = decode_max_parts(page_table.shape[1] * 16)
    for t0 in range(0, T, WIDE_PREFILL_SLICE):
        t1 = min(T, t0 + WIDE_PREFILL_SLICE)
        paged_decode(q[t0:t1], k_cache, v_cache, pt[t0:t1], seq_lens[t0:t1], scale, window, sinks, softcap,
                     k_scale, v_scale, max_parts, out=out[t0:t1])
    return out


_lib.register_signatures({
    "b200_paged_selected_decode": (_lib.i32, [_lib.vp, _lib.vp, _lib.vp, _lib.vp, _lib.i32, _lib.vp, _lib.vp,
                                              _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.i32, _lib.f32, _lib.vp,
                                              _lib.vp]),
})


def paged_selected_decode(q, k_cache, v_cache, page_table, seq_lens, sel, scale, out=None):
    """Decode attention of q [B, H, D] over only the selected token positions
    sel [B, S] int32 (-1 = unused slot) of each row's paged KV
    (csrc/kernels/attention_selected.cu on CUDA, the fp32 re-statement on
    CPU). Positions outside [0, seq_len) are ignored."""
    if not q.is_cuda:
        y = ref.paged_selected_decode_ref(q, k_cache, v_cache, page_table, seq_lens, sel, scale)
        if out is not None:
            out.copy_(y)
            return out
        return y
    B, H, D = q.shape
    KVH = k_cache.shape[1]
    q = q.contiguous()
    sel = sel.to(torch.int32).contiguous()
    if out is None:
        out = torch.empty_like(q)
    _lib.check(_lib.lib().b200_paged_selected_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                                     page_table.data_ptr(), page_table.shape[1], seq_lens.data_ptr(),
                                                     sel.data_ptr(), sel.shape[1], B, H, KVH, D, float(scale),
                                                     out.data_ptr(), _lib.stream_ptr(q.device)),
               "paged_selected_decode")
    _lib.count(1)
    return out
