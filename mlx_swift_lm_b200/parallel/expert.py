"""Expert parallelism (EP): each rank owns E / world whole experts of every
MoE layer; routed token rows travel to the owning rank and the expert outputs
travel back.

The reference has no expert parallelism: its tensor-parallel models
channel-split every expert across ranks (the SwitchGLU of
MLXLMCommon/SwitchLayers.swift:478 under the TP plans of its distributed
models). This module adds it as a first-class feature.

Two exchange implementations with one interface (:meth:`ExpertParallel.moe`):

``fused`` (CUDA): the kernels of csrc/kernels/ep.cu over a symmetric-memory
    buffer (CUDA IPC mappings of every rank's buffer). The router top-k runs
    inside the dispatch kernel, which stores each routed row straight into the
    owner's receive buffer over NVLink; the owner runs the MoE sort, gather
    and grouped tcgen05 GEMMs on its receive slots and stores each output row
    back into the source's return buffer; the combine kernel sums the
    weighted outputs. No host synchronisation, so it captures into the decode
    CUDA graph.
``a2a``: ``torch.distributed.all_to_all_single`` of the counts, rows and
    expert ids (NCCL on GPUs, gloo on CPU); the library baseline and the CPU
    test path.

:class:`ExpertParallelDecoderLM` is the model side: attention and the dense
parts are data-parallel over the rows of a step (each rank computes its
contiguous share of the batch against its own KV pages), MoE layers are
expert-parallel, and the step's logits are all-gathered so that every rank
samples the same tokens. Every rank runs the same scheduler on the same
requests, so all ranks take the same steps with the same MoE layers in the
same order -- the lockstep the flag epochs rely on -- with no per-step
agreement messages.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .. import ops
from ..models.batch import ForwardBatch
from ..models.decoder import DecoderLM
from ..ops import _lib
from ..ops.linear import num_sms
from ..ops.qlinear import QuantizedWeight
from .pipeline import split_rows
from .symm import MAX_RANKS, PHASES_PER_STEP, _align, close_symmetric, open_symmetric

_lib.register_signatures({
    "b200_ep_ctx_size": (_lib.i32, []),
    "b200_ep_route_dispatch": (_lib.i32, [_lib.vp, _lib.i32, _lib.vp, _lib.i32, _lib.i32, _lib.i32, _lib.i32,
                                          _lib.vp, _lib.vp, _lib.vp, _lib.vp, _lib.vp]),
    "b200_ep_prepare": (_lib.i32, [_lib.vp, _lib.i32, _lib.vp, _lib.vp]),
    "b200_ep_return": (_lib.i32, [_lib.vp, _lib.i32, _lib.vp, _lib.vp, _lib.vp, _lib.i32, _lib.vp]),
    "b200_ep_combine": (_lib.i32, [_lib.vp, _lib.i32, _lib.vp, _lib.vp, _lib.vp, _lib.i32, _lib.i32, _lib.vp,
                                   _lib.vp]),
}, status_tags=("ep",))

EP_PADS = 4


class EpCtxStruct(C.Structure):
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("base", C.c_void_p * MAX_RANKS),
                ("pads_off", C.c_uint64), ("rx_off", C.c_uint64), ("rmeta_off", C.c_uint64),
                ("rcnt_off", C.c_uint64), ("ret_off", C.c_uint64), ("cap", C.c_int), ("hidden", C.c_int),
                ("experts_local", C.c_int), ("num_experts", C.c_int), ("step_ptr", C.c_void_p),
                ("ticket", C.c_void_p), ("cnt", C.c_void_p)]


def _num_experts(W) -> int:
    return W.num_experts if isinstance(W, QuantizedWeight) else W.shape[0]


class ExpertParallel:
    """Expert-parallel exchange for one group of `world` ranks.

    `max_tokens` bounds the tokens one rank feeds into one MoE call; the
    receive buffers hold ``world * max_tokens * min(k, E_local)`` rows."""

    def __init__(self, num_experts: int, top_k: int, hidden: int, rank: int = 0, world: int = 1, group=None,
                 device="cpu", max_tokens: int = 256, impl: str = "fused"):
        assert num_experts % world == 0, "experts must divide across EP ranks"
        assert world <= MAX_RANKS
        self.E, self.k, self.H = num_experts, top_k, hidden
        self.rank, self.world, self.group = rank, world, group
        self.E_local = num_experts // world
        self.lo, self.hi = rank * self.E_local, (rank + 1) * self.E_local
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        self.kk = min(top_k, self.E_local)  # pairs of one token that can land on one owner
        self.impl = impl if self.device.type == "cuda" else "a2a"
        self.phase = 0
        self.local_ptr, self.peer_ptrs = None, []
        if self.impl == "fused":
            self._open_fused()

    # ------------------------------------------------------------------ fused buffers
    def _open_fused(self):
        L = _lib.lib()
        assert L.b200_ep_ctx_size() == C.sizeof(EpCtxStruct), "EpCtx layout mismatch"
        w, H = self.world, self.H
        self.cap_max = self.max_tokens * self.kk
        rows = w * self.cap_max
        self.pads_off = 0
        self.rx_off = _align(EP_PADS * MAX_RANKS * 4)
        self.rmeta_off = _align(self.rx_off + rows * H * 2)
        self.rcnt_off = _align(self.rmeta_off + rows * 4)
        self.ret_off = _align(self.rcnt_off + MAX_RANKS * 4)
        self.nbytes = _align(self.ret_off + rows * H * 2)
        self.local_ptr, self.peer_ptrs = open_symmetric(self.group, self.rank, w, self.device, self.nbytes)
        dev = self.device
        self.step = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ticket = torch.zeros(2, dtype=torch.int32, device=dev)
        self.cnt = torch.zeros(MAX_RANKS, dtype=torch.int32, device=dev)
        s = EpCtxStruct()
        s.rank, s.world = self.rank, w
        for j in range(MAX_RANKS):
            s.base[j] = self.peer_ptrs[j] if j < w else 0
        s.pads_off, s.rx_off, s.rmeta_off, s.rcnt_off, s.ret_off = (self.pads_off, self.rx_off, self.rmeta_off,
                                                                    self.rcnt_off, self.ret_off)
        s.cap, s.hidden, s.experts_local, s.num_experts = self.cap_max, H, self.E_local, self.E
        s.step_ptr, s.ticket, s.cnt = self.step.data_ptr(), self.ticket.data_ptr(), self.cnt.data_ptr()
        self.ctx = s
        self._ctx_by_cap = {}
        if w > 1:
            dist.barrier(group=self.group)

    def _ctx(self, cap: int):
        """Context blob with the receive layout of `cap` rows per source (the
        same on every rank of a call)."""
        p = self._ctx_by_cap.get(cap)
        if p is None:
            s = EpCtxStruct.from_buffer_copy(self.ctx)
            s.cap = cap
            p = (s, C.cast(C.pointer(s), C.c_void_p))
            self._ctx_by_cap[cap] = p
        return p[1]

    def close(self):
        """Unmap the peers' buffers, then (after every rank did) free ours."""
        if self.local_ptr is not None:
            torch.cuda.synchronize(self.device)
            close_symmetric(self.rank, None, self.peer_ptrs)
            if self.world > 1:
                dist.barrier(group=self.group)
            close_symmetric(self.rank, self.local_ptr, [])
            self.local_ptr, self.peer_ptrs = None, []

    # ------------------------------------------------------------------ step bookkeeping
    def begin_step(self):
        """Advance the device step counter (outside CUDA graphs; every rank,
        once per forward) and restart the phase count."""
        self.phase = 0
        if self.impl == "fused":
            # a device-side increment: stream-ordered, so a host that runs
            # steps ahead of the device cannot skip or repeat an epoch
            self.step.add_(1)

    def _next_phase(self) -> int:
        p = self.phase
        self.phase += 1
        assert self.phase < PHASES_PER_STEP
        return p

    # ------------------------------------------------------------------ MoE layer
    def moe(self, h, logits, experts_gu, experts_d, *, epi="swiglu", mode="softmax_topk", norm_topk=True,
            gu_bias=None, d_bias=None, tokens_max: int | None = None):
        """Routed-expert output [T, H] of this rank's tokens `h` [T, H] with
        router logits [T, E] fp32; `experts_gu` / `experts_d` hold this rank's
        E_local experts. `tokens_max` is the largest T of any rank in this call
        (the same value on every rank; default `max_tokens`)."""
        assert _num_experts(experts_gu) == self.E_local
        if mode not in ("softmax_topk", "topk_softmax"):
            raise NotImplementedError(f"expert parallelism serves softmax routers, not {mode!r}")
        if self.impl == "fused":
            return self._moe_fused(h, logits, experts_gu, experts_d, epi, mode, norm_topk, gu_bias, d_bias,
                                   tokens_max or self.max_tokens)
        return self._moe_a2a(h, logits, experts_gu, experts_d, epi, mode, norm_topk, gu_bias, d_bias)

    def _moe_fused(self, h, logits, Wgu, Wd, epi, mode, norm_topk, gu_bias, d_bias, tokens_max):
        from ..ops import moe as moe_ops

        T, H = h.shape
        k = self.k
        assert T <= tokens_max <= self.max_tokens, f"{T} tokens > EP capacity {self.max_tokens}"
        cap = tokens_max * self.kk
        ctx = self._ctx(cap)
        phase = self._next_phase()
        dev = h.device
        L = _lib.lib()
        st = _lib.stream_ptr(dev)
        hc = h.contiguous()
        lg = logits.float().contiguous()
        ids = torch.empty(max(T, 1), k, dtype=torch.int32, device=dev)
        w = torch.empty(max(T, 1), k, dtype=torch.float32, device=dev)
        slots = torch.empty(max(T, 1), k, dtype=torch.int32, device=dev)
        _lib.check(L.b200_ep_route_dispatch(ctx, phase, lg.data_ptr(), T, k, 1 if mode == "topk_softmax" else 0,
                                            1 if norm_topk else 0, hc.data_ptr(), ids.data_ptr(), w.data_ptr(),
                                            slots.data_ptr(), st), "ep_route_dispatch")
        # ---- owner side: every slot of every source
        P = self.world * cap
        El = self.E_local
        ids_local = torch.empty(P, dtype=torch.int32, device=dev)
        _lib.check(L.b200_ep_prepare(ctx, phase, ids_local.data_ptr(), st), "ep_prepare")
        if isinstance(Wgu, QuantizedWeight):
            N2 = Wgu.shape[0] // El
            F = Wd.shape[1]
        else:
            N2, F = Wgu.shape[1], Wd.shape[2]
        BN = moe_ops.chunk_rows(tokens_max * k, El)
        max_chunks = (P + BN - 1) // BN + El
        perm = torch.empty(P, dtype=torch.int32, device=dev)
        pos = torch.empty(P, dtype=torch.int32, device=dev)
        chunks = torch.empty(max_chunks * 3, dtype=torch.int32, device=dev)
        n_chunks = torch.empty(1, dtype=torch.int32, device=dev)
        xs = torch.empty(P, H, dtype=h.dtype, device=dev)
        gu = torch.empty(P, F, dtype=h.dtype, device=dev)
        ys = torch.empty(P, H, dtype=h.dtype, device=dev)
        _lib.check(L.b200_moe_sort(ids_local.data_ptr(), P, El, BN, max_chunks, perm.data_ptr(), pos.data_ptr(),
                                   chunks.data_ptr(), n_chunks.data_ptr(), st), "moe_sort")
        _lib.check(L.b200_moe_gather(self.local_ptr + self.rx_off, H, perm.data_ptr(), P, 1, xs.data_ptr(), 0, st),
                   "moe_gather")
        moe_ops._grouped(L, xs, P, H, Wgu, El, N2, gu, F, gu_bias, moe_ops._EPI[epi], chunks, n_chunks, max_chunks,
                         BN, st, "gate/up")
        moe_ops._grouped(L, gu, P, F, Wd, El, H, ys, H, d_bias, 0, chunks, n_chunks, max_chunks, BN, st, "down")
        _lib.check(L.b200_ep_return(ctx, phase, ys.data_ptr(), pos.data_ptr(), ids_local.data_ptr(),
                                    num_sms(dev), st), "ep_return")
        # ---- source side
        out = torch.empty(T, H, dtype=h.dtype, device=dev)
        _lib.check(L.b200_ep_combine(ctx, phase, ids.data_ptr(), w.data_ptr(), slots.data_ptr(), T, k,
                                     out.data_ptr(), st), "ep_combine")
        _lib.count(8)
        return out

    def _moe_a2a(self, h, logits, Wgu, Wd, epi, mode, norm_topk, gu_bias, d_bias):
        from ..ops import moe as moe_ops

        T, H = h.shape
        k, El, world = self.k, self.E_local, self.world
        w, ids = moe_ops.route_topk(logits, k, mode, norm_topk)
        ids = ids.long()
        owner = (ids // El).reshape(-1)
        order = torch.argsort(owner, stable=True)
        send_counts = torch.bincount(owner, minlength=world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        send_rows = h.index_select(0, order // k).contiguous()
        send_ids = (ids.reshape(-1)[order] - owner[order] * El).to(torch.int64)
        recv_rows = torch.empty(sum(rc), H, dtype=h.dtype, device=h.device)
        recv_ids = torch.empty(sum(rc), dtype=torch.int64, device=h.device)
        dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids, rc, sc, group=self.group)
        R = recv_rows.shape[0]
        if R:
            ones = torch.ones(R, 1, dtype=torch.float32, device=h.device)
            y = moe_ops.moe_experts(recv_rows, Wgu, Wd, ones, recv_ids[:, None].to(torch.int32 if h.is_cuda
                                                                                    else torch.int64),
                                    epi, gu_bias, d_bias)
        else:
            y = recv_rows
        back = torch.empty(T * k, H, dtype=h.dtype, device=h.device)
        dist.all_to_all_single(back, y.contiguous(), sc, rc, group=self.group)
        ypairs = torch.empty_like(back)
        ypairs[order] = back
        yp = ypairs.view(T, k, H).float()
        out = torch.zeros(T, H, dtype=torch.float32, device=h.device)
        for j in range(k):
            out += w[:, j:j + 1].float() * yp[:, j]
        return out.to(h.dtype)


# ---------------------------------------------------------------------- model side
def _pad_part(fb: ForwardBatch) -> ForwardBatch:
    """One inert decode row (no KV write, empty context) for a rank that has
    no rows in a step; its output is dropped."""
    dev = fb.input_ids.device
    mb = ForwardBatch(input_ids=torch.zeros(1, dtype=torch.int32, device=dev),
                      positions=torch.zeros(1, dtype=torch.int32, device=dev),
                      slots=torch.full((1,), -1, dtype=torch.int64, device=dev), num_decode=1)
    mb.dec_page_table = torch.zeros(1, 1, dtype=torch.int32, device=dev)
    mb.dec_seq_lens = torch.zeros(1, dtype=torch.int32, device=dev)
    mb.dec_max_parts = 1
    mb.pad = True
    return mb


def select_rows(fb: ForwardBatch, rows: list[int]) -> ForwardBatch:
    """Sub-batch of the given rows (ascending row indices: decode rows are
    0..num_decode-1, prefill row j is num_decode + j). ``logit_src`` lists
    the positions in ``fb``'s logit order of the sub-batch's logit rows."""
    nd = fb.num_decode
    pf_cu = fb.pf_cu_q_host or [0]
    dev = fb.input_ids.device
    dec = [r for r in rows if r < nd]
    pfr = [r - nd for r in rows if r >= nd]
    toks = list(dec)
    cu = [0]
    for j in pfr:
        a, b = nd + pf_cu[j], nd + pf_cu[j + 1]
        toks.extend(range(a, b))
        cu.append(cu[-1] + b - a)
    ti = torch.tensor(toks, dtype=torch.int64, device=dev)
    mb = ForwardBatch(input_ids=fb.input_ids[ti], positions=fb.positions[ti], slots=fb.slots[ti],
                      num_decode=len(dec))
    if dec:
        di = torch.tensor(dec, dtype=torch.int64, device=dev)
        mb.dec_page_table = fb.dec_page_table[di]
        mb.dec_seq_lens = fb.dec_seq_lens[di]
        mb.dec_max_parts = fb.dec_max_parts
    if pfr:
        pi = torch.tensor(pfr, dtype=torch.int64, device=dev)
        mb.pf_cu_q_host = cu
        mb.pf_cu_q = torch.tensor(cu, dtype=torch.int32, device=dev)
        mb.pf_pos0 = fb.pf_pos0[pi]
        mb.pf_page_table = fb.pf_page_table[pi]
    if fb.logit_idx is not None:
        gl = fb.logit_idx_host if fb.logit_idx_host is not None else fb.logit_idx.tolist()
        where = {t: i for i, t in enumerate(toks)}
        sel = [(where[t], g) for g, t in enumerate(gl) if t in where]
        mb.logit_idx_host = [a for a, _ in sel]
        mb.logit_idx = torch.tensor(mb.logit_idx_host, dtype=torch.int64, device=dev)
        mb.logit_src = [g for _, g in sel]
    else:
        mb.logit_src = toks
    mb.pad = False
    return mb


def shard_rows(fb: ForwardBatch, n: int) -> list[ForwardBatch]:
    """Exactly n shards of a forward batch: the rows of each rank when
    ``fb.row_ranks`` is set (rows stay with the rank that holds their KV),
    else contiguous row ranges balanced by tokens. Shards without rows are
    single padding rows (attribute ``pad``)."""
    R = fb.num_decode + len(fb.pf_cu_q_host or [0]) - 1
    if fb.row_ranks is not None:
        groups = [[i for i in range(R) if fb.row_ranks[i] == r] for r in range(n)]
    else:
        parts = split_rows(fb, n)
        groups, i = [], 0
        for p in parts:
            k = p.num_decode + len(p.pf_cu_q_host or [0]) - 1
            groups.append(list(range(i, i + k)))
            i += k
        groups += [[] for _ in range(n - len(groups))]
    return [select_rows(fb, g) if g else _pad_part(fb) for g in groups]


def _out_rows(p: ForwardBatch) -> int:
    if p.logit_idx is None:
        return p.num_tokens
    return len(p.logit_idx_host) if p.logit_idx_host is not None else int(p.logit_idx.numel())


class ExpertParallelDecoderLM(DecoderLM):
    """A decoder whose MoE layers run expert-parallel over `ep` and whose
    attention / dense parts are data-parallel over the rows of each step.
    Built from the full random-init weights (same seed on every rank), each
    rank keeps its E / world experts of every MoE layer."""

    def __init__(self, cfg, ep: ExpertParallel, device="cpu", dtype=torch.float32):
        super().__init__(cfg, device, dtype)
        self.ep = ep
        self._tokens_max = None

    @property
    def dp_world(self) -> int:
        """Ranks the rows of a step are split across (each keeps its rows' KV)."""
        return self.ep.world

    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True, keep_layers=None):
        super().init_random(seed, std, with_embeddings, keep_layers)
        return self.localize_experts()

    def localize_experts(self):
        """Keep this rank's experts [lo, hi) of every MoE layer."""
        lo, hi = self.ep.lo, self.ep.hi
        for L in self.layers:
            if not L.moe:
                continue
            if _num_experts(L.experts_gu) == self.ep.E_local:
                continue
            for name in ("experts_gu", "experts_d", "experts_gu_b", "experts_d_b"):
                t = getattr(L, name)
                if t is None:
                    continue
                if isinstance(t, QuantizedWeight):
                    raise ValueError("localize experts before quantising them")
                setattr(L, name, t[lo:hi].contiguous())
        return self

    # ------------------------------------------------------------------ pieces
    def _moe(self, L, h):
        cfg = self.cfg
        if self.ep.world == 1 and _num_experts(L.experts_gu) == self.ep.E:
            return super()._moe(L, h)
        logits = ops.gemm(h, L.router, epi="f32", bias=L.router_b)
        out = self.ep.moe(h, logits, L.experts_gu, L.experts_d, epi=cfg.glu_epi, mode=cfg.router_mode,
                          norm_topk=cfg.norm_topk_prob, gu_bias=L.experts_gu_b, d_bias=L.experts_d_b,
                          tokens_max=self._tokens_max)
        if L.shared_gu is not None:
            s = ops.gemm(ops.gemm(h, L.shared_gu, epi=cfg.glu_epi), L.shared_d)
            if L.shared_gate is not None:
                s = (torch.sigmoid(ops.gemm(h, L.shared_gate, epi="f32")) * s.float()).to(s.dtype)
            out = (out.float() + s.float()).to(out.dtype)
        return out

    def begin_step(self):
        self.ep.begin_step()

    def _capturing(self) -> bool:
        return self.device.type == "cuda" and torch.cuda.is_current_stream_capturing()

    def _gather_rows(self, local: torch.Tensor, counts: list[int]) -> torch.Tensor:
        """All-gather row blocks of different lengths (rank order)."""
        world = self.ep.world
        nmax = max(counts)
        buf = local.new_zeros((nmax,) + tuple(local.shape[1:]))
        buf[:local.shape[0]] = local
        if dist.get_backend(self.ep.group) == "nccl":
            allb = local.new_empty((world * nmax,) + tuple(local.shape[1:]))
            dist.all_gather_into_tensor(allb, buf, group=self.ep.group)
            blocks = list(allb.view((world, nmax) + tuple(local.shape[1:])))
        else:
            blocks = [torch.empty_like(buf) for _ in range(world)]
            dist.all_gather(blocks, buf, group=self.ep.group)
        return torch.cat([b[:c] for b, c in zip(blocks, counts) if c], 0)

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        ep = self.ep
        if ep.world == 1:
            if not self._capturing():
                self.begin_step()
            self._tokens_max = fb.num_tokens
            return super().forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        assert inputs_embeds is None and not return_residual, "EP models are whole (no pipeline stages)"
        if not self._capturing():
            self.begin_step()
        parts = shard_rows(fb, ep.world)
        self._tokens_max = max(p.num_tokens for p in parts)
        mine = parts[ep.rank]
        res = DecoderLM.forward(self, mine, kv, return_hidden=return_hidden, return_both=return_both)
        counts = [0 if p.pad else _out_rows(p) for p in parts]
        src = [g for p in parts if not p.pad for g in p.logit_src]
        inv = torch.empty(len(src), dtype=torch.int64)
        inv[torch.tensor(src, dtype=torch.int64)] = torch.arange(len(src))
        inv = inv.to(self.device)

        def gather(t):
            return self._gather_rows(t if not mine.pad else t[:0], counts).index_select(0, inv)

        if return_both:
            return gather(res[0]), gather(res[1])
        return gather(res)

    def forward_greedy_both(self, fb: ForwardBatch, kv):
        """Greedy tokens and hiddens of the logit rows: each rank takes the
        argmax of its own rows, so only tokens and hiddens are gathered
        (not [rows, vocab] logits)."""
        ep = self.ep
        if ep.world == 1:
            return super().forward_greedy_both(fb, kv)
        if not self._capturing():
            self.begin_step()
        parts = shard_rows(fb, ep.world)
        self._tokens_max = max(p.num_tokens for p in parts)
        mine = parts[ep.rank]
        logits, h = DecoderLM.forward(self, mine, kv, return_both=True)
        tok = ops.argmax(logits)
        counts = [0 if p.pad else _out_rows(p) for p in parts]
        src = [g for p in parts if not p.pad for g in p.logit_src]
        inv = torch.empty(len(src), dtype=torch.int64)
        inv[torch.tensor(src, dtype=torch.int64)] = torch.arange(len(src))
        inv = inv.to(self.device)
        if mine.pad:
            tok, h = tok[:0], h[:0]
        return (self._gather_rows(tok, counts).index_select(0, inv),
                self._gather_rows(h, counts).index_select(0, inv))

    def forward_decode_tokens(self, fb: ForwardBatch, kv, out: torch.Tensor, out2=None, flags=None):
        """Greedy tokens of a pure-decode batch whose row count is a multiple
        of the EP world (decode graph buckets): rank r computes rows
        [r * S, (r + 1) * S) and the tokens are all-gathered."""
        ep = self.ep
        B = fb.num_tokens
        if ep.world == 1 or B % ep.world or fb.num_decode != B:
            logits = self.forward(fb, kv)
            return ops.argmax(logits, out=out, out2=out2, flags=flags)
        if not self._capturing():
            self.begin_step()
        S = B // ep.world
        a, b = ep.rank * S, (ep.rank + 1) * S
        mine = ForwardBatch(input_ids=fb.input_ids[a:b], positions=fb.positions[a:b], slots=fb.slots[a:b],
                            num_decode=S, dec_page_table=fb.dec_page_table[a:b], dec_seq_lens=fb.dec_seq_lens[a:b],
                            dec_max_parts=fb.dec_max_parts)
        self._tokens_max = S
        logits = DecoderLM.forward(self, mine, kv)
        tok = ops.argmax(logits)
        dist.all_gather_into_tensor(out[:B], tok.to(out.dtype).contiguous(), group=ep.group)
        if out2 is not None:
            out2[:B].copy_(out[:B])
        return out
