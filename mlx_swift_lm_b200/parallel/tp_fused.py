"""Fused tensor-parallel decode forward over symmetric memory.

Per layer (the residual stream x and the normed rows h are replicated on
every rank; one cross-rank synchronisation per row-parallel projection):

    q, K/V = GEMM(h, Wqkv_r) + qk-norm + RoPE + paged K/V append (local)
    attn   = paged attention on the rank's heads (all rows)
    GEMM_RS(attn, Wo_r)        the epilogue writes its fp32 partial rows into
                               every rank's inbox, the last CTA signals
    x, h   = combine_all(ln2)  wait for every rank's partials, sum them in
                               rank order (identical on every rank), add to x,
                               RMSNorm into h (local, nothing pushed)
    gu     = GEMM(h, Wgu_r, SwiGLU) (local)
    GEMM_RS(gu, Wd_r); x, h = combine_all(ln1 of the next layer / final norm)

Sending every rank all partials costs (world - 1) x rows x hidden x 4 bytes
per projection per rank (0.5-3.5 MB at 64 rows of 4096 for 2-8 ranks), and
saves the second exchange of a reduce-scatter + all-gather pair (a push of
normed rows and its flag round trip) per projection.

The head is vocabulary-parallel (rank r holds rows [r*V/N, (r+1)*V/N) of the
LM head) and the token is a cross-rank split argmax, so every rank ends the
step with identical tokens. Parity: the reference's 2-rank tensor-parallel
path (Gemma4TensorParallel.swift, TensorParallelSwitchLinear.swift,
vocab-split head Gemma4Text.swift:2213) generalised to N ranks, with the
collectives fused into the GEMMs instead of injected closures.
"""
from __future__ import annotations

import os
import warnings

import torch

from .. import ops
from ..ops import _lib
from ..ops.linear import num_sms
from .symm import SymmetricComm

_EPI = {"none": 0, "swiglu": 1, "f32": 2, "geglu": 4, "swiglu_oai": 5}


def nvls_buffer(group, shape, dev):
    """A bf16 buffer bound to an NVLink multicast object over `group` (torch
    symmetric memory): (tensor, multicast address of its first element), or
    None where the system offers no multicast. Collective: every rank of the
    group calls it."""
    try:
        import torch.distributed._symmetric_memory as symm_mem

        buf = symm_mem.empty(shape, dtype=torch.bfloat16, device=dev)
        hdl = symm_mem.rendezvous(buf, group.group_name)
        if not hdl.multicast_ptr:
            return None
        buf.zero_()
        rank = torch.distributed.get_rank(group)
        return buf, hdl, int(hdl.multicast_ptr) + (buf.data_ptr() - int(hdl.buffer_ptrs[rank]))
    except Exception as e:  # no symmetric-memory backend or no NVLS
        warnings.warn(f"NVLS multicast buffer unavailable: {e}")
        return None


def rows_per_rank(T: int, world: int) -> int:
    r = (T + world - 1) // world
    return max(8, (r + 7) // 8 * 8)


class FusedTP:
    def __init__(self, model, max_rows: int):
        tp = model.tp
        self.m = model
        self.world, self.rank = tp.world, tp.rank
        self.rpr = rows_per_rank(max_rows, self.world)
        self.M_pad = self.world * self.rpr
        assert self.M_pad in (16, 32, 64, 128, 256), f"fused TP supports up to 256 padded rows, got {self.M_pad}"
        cfg = model.cfg
        self.comm = SymmetricComm(tp.group, tp.rank, tp.world, model.device, cfg.hidden_size, self.rpr,
                                  max_rows=self.M_pad)
        dev, dt = model.device, model.dtype
        self.x_local = torch.zeros(self.rpr, cfg.hidden_size, dtype=dt, device=dev)
        V = cfg.vocab_size
        assert V % self.world == 0, "vocabulary must split evenly across ranks"
        self.V_local = V // self.world
        self.head = model.lm_head[self.rank * self.V_local:(self.rank + 1) * self.V_local]
        self.qkv = torch.empty(self.M_pad, (model.H + 2 * model.KVH) * model.D, dtype=dt, device=dev)
        # replicated residual rows and their normed copy (the local GEMMs' input)
        self.x = torch.zeros(self.M_pad, cfg.hidden_size, dtype=dt, device=dev)
        self.h = torch.zeros(self.M_pad, cfg.hidden_size, dtype=dt, device=dev)
        self.gu = torch.empty(self.M_pad, model.F, dtype=dt, device=dev)
        self.logits = torch.empty(self.M_pad, self.V_local, dtype=torch.float32, device=dev)
        self.sms = num_sms(dev)
        # from 4 ranks up the partial rows cross NVLink as bf16 (half the bytes; summed in fp32)
        self.rs_mode = 2 if self.world >= 4 else 1
        # B200LM_TP_NVLS=1: each rank stores its bf16 partials locally and the
        # combine reads their sum through the NVSwitch (multimem.ld_reduce)
        self.nvls = None
        if os.environ.get("B200LM_TP_NVLS", "0") == "1":
            self.nvls = nvls_buffer(tp.group, (2, self.M_pad, cfg.hidden_size), dev)
            if self.nvls is not None:
                self.rs_mode = 3

    # ------------------------------------------------------------------ primitives
    def _publish(self, w, has_delta, rs):
        c = self.comm
        p = c.next_phase()
        par = c.ag_count & 1
        c.ag_count += 1
        _lib.check(_lib.lib().b200_tp_combine_norm(c.ctx_ptr, rs[0] if rs else 0, rs[1] if rs else 0, p, par,
                                                   self.x_local.data_ptr(), w.data_ptr(), float(self.m.cfg.rms_norm_eps),
                                                   1 if has_delta else 0, _lib.stream_ptr(self.m.device)),
                   "tp_combine_norm")
        _lib.count(1)
        return (p, par)

    def _gemm_ag(self, ag, T, W, out, epi="none", bias=None):
        c = self.comm
        K = W.shape[1]
        _lib.check(_lib.lib().b200_gemm_bf16_ag(c.ctx_ptr, ag[0], ag[1], T, K, W.data_ptr(), W.shape[0], W.stride(0),
                                                out.data_ptr(), out.stride(0), _lib.ptr(bias), _EPI[epi], self.sms, 0,
                                                _lib.stream_ptr(self.m.device)), "gemm_ag")
        _lib.count(1)
        return out

    def _gemm_rs(self, X, T, W, bias=None, rs_all=False):
        c = self.comm
        p = c.next_phase()
        par = c.rs_count & 1
        c.rs_count += 1
        _lib.check(_lib.lib().b200_gemm_bf16_rs(c.ctx_ptr, p, par, X.data_ptr(), T, X.shape[1], X.stride(0),
                                                W.data_ptr(), W.shape[0], W.stride(0),
                                                _lib.ptr(bias) if self.rank == 0 else None, self.sms, 0,
                                                self.rs_mode if rs_all else 0,
                                                self.nvls[0].data_ptr() if self.rs_mode == 3 else None,
                                                _lib.stream_ptr(self.m.device)), "gemm_rs")
        _lib.count(1)
        return (p, par)

    def _combine_all(self, rs, T, w):
        """x += rank-ordered sum of every rank's partials (rs = None: no delta); h = RMSNorm(x) * w."""
        c = self.comm
        _lib.check(_lib.lib().b200_tp_combine_all(c.ctx_ptr, rs[0] if rs else 0, rs[1] if rs else 0,
                                                  self.x.data_ptr(), w.data_ptr(), float(self.m.cfg.rms_norm_eps),
                                                  self.h.data_ptr(), T, 1 if rs else 0,
                                                  1 if self.rs_mode == 2 else 0,
                                                  self.nvls[2] if self.rs_mode == 3 else None,
                                                  _lib.stream_ptr(self.m.device)), "tp_combine_all")
        _lib.count(1)

    # ------------------------------------------------------------------ forward
    def decode_tokens(self, fb, kv, out, out2=None):
        """Pure-decode step: writes the greedy tokens of fb's rows into `out`."""
        m, cfg, c = self.m, self.m.cfg, self.comm
        T = fb.num_tokens
        assert T <= self.M_pad
        c.phase = 0
        L = _lib.lib()
        st = _lib.stream_ptr(m.device)
        ops.embedding(fb.input_ids, m.embed, cfg.embed_scale, out=self.x[:T])
        self._combine_all(None, T, m.layers[0].ln1)
        h = self.h[:T]
        for li, Lw in enumerate(m.layers):
            kc, vc = kv.layer(li)
            cs, rd = m.rope_for(li)
            if m._fused_qkv_rope(Lw, h, fb, rd):
                q = ops.gemm_qkv_rope(h, Lw.wqkv, Lw.bqkv, fb.positions, fb.slots, cs, Lw.q_norm, Lw.k_norm,
                                      cfg.rms_norm_eps, kc, vc, m.H, m.KVH, kv.k_scale(li), kv.v_scale(li))
            else:
                qkv = ops.gemm(h, Lw.wqkv, bias=Lw.bqkv, out=self.qkv[:T])
                q = ops.qk_norm_rope_kv(qkv, fb.positions, fb.slots, cs, rd, cfg.rope_interleaved,
                                        Lw.q_norm, Lw.k_norm, cfg.rms_norm_eps, kc, vc, m.H, m.KVH, m.D,
                                        kv.k_scale(li), kv.v_scale(li))
            attn = ops.paged_decode(q, kc, vc, fb.dec_page_table, fb.dec_seq_lens, cfg.scale, cfg.window(li),
                                    Lw.sinks, cfg.attn_logit_softcap, kv.k_scale(li), kv.v_scale(li),
                                    fb.dec_max_parts)
            rs = self._gemm_rs(attn.view(T, m.H * m.D), T, Lw.wo, Lw.bo, rs_all=True)
            self._combine_all(rs, T, Lw.ln2)
            ops.gemm(h, Lw.wgu, epi=cfg.glu_epi, bias=Lw.bgu, out=self.gu[:T])
            rs = self._gemm_rs(self.gu[:T], T, Lw.wd, Lw.bd, rs_all=True)
            nxt = m.layers[li + 1].ln1 if li + 1 < len(m.layers) else m.norm
            self._combine_all(rs, T, nxt)
        ops.gemm(h, self.head, epi="f32", out=self.logits[:T])
        p = c.next_phase()
        par = c.arg_count & 1
        c.arg_count += 1
        _lib.check(L.b200_tp_argmax(c.ctx_ptr, p, par, self.logits.data_ptr(), self.logits.stride(0), T,
                                    self.V_local, self.rank * self.V_local, out.data_ptr(), _lib.ptr(out2), st),
                   "tp_argmax")
        _lib.count(2)
        return out
