"""CUDA-graph decode runner: one captured graph per decode batch bucket.

A pure-decode step of B rows replays the graph of the smallest bucket >= B
(padding rows write no KV: slot -1, length 0). All per-step inputs live in one
packed device buffer that a single host->device copy refreshes from a
double-buffered pinned staging area; the sampled tokens land in a shared
device buffer and are copied back to pinned memory asynchronously. Input ids
of a chained step are gathered on the device from the previous step's output
(``gather_tokens``), so step N+1 can be launched before the host has read
step N's tokens. This replaces the reference's MLX ``compile`` traces of the
decode step (MLXLMCommon/CompiledTrace.swift:51, CompiledDecodeSegments.swift:10).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..models.batch import ForwardBatch
from ..ops import _lib
from ..ops.attention import SCRATCH, decode_max_parts, merge_counters
from .sampler import row_key

PENDING = -1


class DecodeGraphRunner:
    def __init__(self, engine):
        self.eng = engine
        self.model = engine.model
        self.dev = engine.device
        mc = engine.cfg.scheduler.max_concurrent_requests
        bk = sorted(b for b in engine.cfg.graph_buckets if b <= max(mc, 1))
        if not bk or bk[-1] < mc:
            bk.append(mc)
        # models that split rows across data-parallel ranks take rank r's rows
        # in the slice [r * B / world, (r + 1) * B / world) of a bucket of B
        self.dp = getattr(self.model, "dp_world", 1)
        if self.dp > 1:
            bk = sorted({-(-b // self.dp) * self.dp for b in bk})
        self.buckets = bk
        self.Bmax = bk[-1] + (bk[-1] % 2)
        self.maxp = engine.max_pages
        self.max_parts = decode_max_parts(engine.cfg.max_model_len)
        B, P = self.Bmax, self.maxp
        # packed int32 layout: pos | seq_lens | src | host_ids | page_table | slots(int64) | state slots |
        # sampling: rng keys (int64) | rng steps (int64) | temperature f32 | top_k | top_p f32 | min_p f32
        self.o_pos, self.o_sl, self.o_src, self.o_hid, self.o_pt = 0, B, 2 * B, 3 * B, 4 * B
        self.o_slots = 4 * B + B * P
        self.o_slots += self.o_slots % 2
        self.o_ss = self.o_slots + 2 * B
        self.o_key = self.o_ss + B + (self.o_ss + B) % 2
        self.o_step = self.o_key + 2 * B
        self.o_temp = self.o_step + 2 * B
        self.o_topk, self.o_topp, self.o_minp = self.o_temp + B, self.o_temp + 2 * B, self.o_temp + 3 * B
        self.n_i32 = self.o_temp + 4 * B
        # sliding-window ring layers: ring slots (int64) | ring page table
        self.ring = engine.kv.ring_pages > 0
        if self.ring:
            self.o_rslots = self.n_i32 + self.n_i32 % 2
            self.o_rpt = self.o_rslots + 2 * B
            self.n_i32 = self.o_rpt + B * P
        # per-row batched-LoRA adapter slot (-1 = none)
        self.o_lora = self.n_i32
        self.n_i32 += B
        self.rec = engine.kv.rec
        self.packed = torch.zeros(self.n_i32, dtype=torch.int32, device=self.dev)
        self.staging = [torch.zeros(self.n_i32, dtype=torch.int32).pin_memory() for _ in range(2)]
        self.staging_ev = [None, None]
        self.slot_k = 0
        self.pos = self.packed[self.o_pos:self.o_pos + B]
        self.sl = self.packed[self.o_sl:self.o_sl + B]
        self.src = self.packed[self.o_src:self.o_src + B]
        self.hid = self.packed[self.o_hid:self.o_hid + B]
        self.pt = self.packed[self.o_pt:self.o_pt + B * P].view(B, P)
        self.slots = self.packed[self.o_slots:self.o_slots + 2 * B].view(torch.int64)
        self.ss = self.packed[self.o_ss:self.o_ss + B]
        self.s_key = self.packed[self.o_key:self.o_key + 2 * B].view(torch.int64)
        self.s_step = self.packed[self.o_step:self.o_step + 2 * B].view(torch.int64)
        self.s_temp = self.packed[self.o_temp:self.o_temp + B].view(torch.float32)
        self.s_topk = self.packed[self.o_topk:self.o_topk + B]
        self.s_topp = self.packed[self.o_topp:self.o_topp + B].view(torch.float32)
        self.s_minp = self.packed[self.o_minp:self.o_minp + B].view(torch.float32)
        if self.ring:
            self.rslots = self.packed[self.o_rslots:self.o_rslots + 2 * B].view(torch.int64)
            self.rpt = self.packed[self.o_rpt:self.o_rpt + B * P].view(B, P)
        self.lslots = self.packed[self.o_lora:self.o_lora + B]
        # sampled rows (temperature / top-k / top-p / min-p) run a second graph per bucket
        # whose last kernel draws from the logits instead of taking the argmax
        self.sampling = self._supports_sampling()
        self.sgraphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.ids = torch.zeros(B, dtype=torch.int32, device=self.dev)
        self.out = torch.zeros(B, dtype=torch.int32, device=self.dev)
        # non-finite-logit flag per row, read back with the tokens
        self.flags = torch.zeros(B, dtype=torch.int32, device=self.dev)
        self.host_out = [torch.zeros(B, dtype=torch.int32).pin_memory() for _ in range(4)]
        self.host_flags = [torch.zeros(B, dtype=torch.int32).pin_memory() for _ in range(4)]
        self.out_k = 0
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        # rows with batched LoRA adapters: unfused projections plus adapter deltas
        self.lgraphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.lsgraphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.pool = None
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.launches_per_replay: dict[int, int] = {}
        self._reserved = False
        # chained-decode input ids: the gather_tokens kernel, or a model-supplied
        # callable(prev_out, src, host_ids, ids, B) (the PyTorch baseline)
        self.gather_fn = None

    # ------------------------------------------------------------------ capture
    def _reserve(self):
        if self._reserved:
            return
        m = self.model
        H, D = m.attn_scratch_dims()
        SCRATCH.get(self.dev, "dec_acc", self.Bmax * H * self.max_parts * D)
        SCRATCH.get(self.dev, "dec_ml", self.Bmax * H * self.max_parts * 2)
        merge_counters(self.dev, self.Bmax * max(m.KVH, 1))
        ops.WORKSPACE.reserve(self.dev, 512 << 20)
        self._reserved = True

    def _fb(self, B):
        fb = ForwardBatch(input_ids=self.ids[:B], positions=self.pos[:B], slots=self.slots[:B], num_decode=B,
                          dec_page_table=self.pt[:B], dec_seq_lens=self.sl[:B], dec_max_parts=self.max_parts,
                          state_slots=self.ss[:B] if self.rec is not None else None)
        if self.ring:
            fb.ring_slots, fb.ring_dec_page_table = self.rslots[:B], self.rpt[:B]
        return fb

    def _supports_sampling(self) -> bool:
        """Sampled graphs need the full logits on every rank: not the fused TP
        path (vocab-split head), not row-split data-parallel models."""
        m = self.model
        return (self.dp <= 1 and getattr(m, "tp_fused", None) is None and getattr(m, "pp_stages", 1) == 1
                and getattr(m, "graph_sampling", True))

    def _store(self, sampled: bool, lora: bool) -> dict:
        if lora:
            return self.lsgraphs if sampled else self.lgraphs
        return self.sgraphs if sampled else self.graphs

    @staticmethod
    def _key(B, sampled, lora):
        return (("l" if lora else "") + ("s" if sampled else ""), B) if (sampled or lora) else B

    def _body(self, B, sampled=False, lora=False):
        fb = self._fb(B)
        if lora:
            fb.lora_slots = self.lslots[:B]
        if not sampled:
            self.model.forward_decode_tokens(fb, self.eng.kv, self.out[:B], flags=self.flags[:B])
            return
        logits = self.model.forward(fb, self.eng.kv)
        ops.sample(logits, self.s_temp[:B], self.s_topk[:B], self.s_topp[:B], self.s_minp[:B], self.s_key[:B],
                   self.s_step[:B], out=self.out[:B], flags=self.flags[:B])

    def capture(self, B, sampled=False, lora=False):
        self._reserve()
        # inert inputs for warm-up: no KV writes, empty contexts, scratch recurrent state
        if self.rec is not None:
            self.ss.fill_(self.rec.scratch)
        self.slots.fill_(-1)
        if self.ring:
            self.rslots.fill_(-1)
        self.sl.zero_()
        self.pos.zero_()
        self.ids.zero_()
        self.s_temp.zero_()
        cur = torch.cuda.current_stream(self.dev)
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(cur)
        self.lslots.fill_(-1)
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.begin_step()
                self._body(B, sampled, lora)
        cur.wait_stream(s)
        torch.cuda.synchronize(self.dev)
        n0 = _lib.launch_counter[0]
        g = torch.cuda.CUDAGraph()
        self.model.begin_step()  # the capture itself does not run; every replay advances the step first
        with torch.cuda.graph(g, pool=self.pool):
            self._body(B, sampled, lora)
        self.launches_per_replay[self._key(B, sampled, lora)] = _lib.launch_counter[0] - n0
        if self.pool is None:
            self.pool = g.pool()
        self._store(sampled, lora)[B] = g
        torch.cuda.synchronize(self.dev)

    def invalidate(self):
        """Drop every captured graph (buffers they point to are about to move)."""
        for d in (self.graphs, self.sgraphs, self.lgraphs, self.lsgraphs):
            d.clear()
        self._reserved = False

    def capture_all(self):
        for b in reversed(self.buckets):
            if b not in self.graphs:
                self.capture(b)

    # ------------------------------------------------------------------ run
    def bucket(self, n):
        for b in self.buckets:
            if b >= n:
                return b
        return None

    def layout(self, plan):
        """(bucket, buffer position of each plan row), or (None, None)."""
        rows = plan.rows
        if self.dp <= 1:
            return self.bucket(len(rows)), list(range(len(rows)))
        ranks = self.eng._row_ranks(rows)
        per = [0] * self.dp
        for d in ranks:
            per[d] += 1
        Bb = self.bucket(self.dp * max(per))
        if Bb is None:
            return None, None
        S = Bb // self.dp
        nxt = [d * S for d in range(self.dp)]
        pos = []
        for d in ranks:
            pos.append(nxt[d])
            nxt[d] += 1
        return Bb, pos

    def can_run(self, plan) -> bool:
        if self.layout(plan)[0] is None:
            return False
        for r in plan.rows:
            if len(r.state.seq.pages) > self.maxp:
                return False
        return True

    def chainable(self, prev, plan) -> bool:
        return True

    def launch(self, plan, chained_from=None):
        rows = plan.rows
        n = len(rows)
        Bb, where = self.layout(plan)
        sampled = any(not r.state.req.sampling.greedy for r in rows)
        lora = any(r.state.extra.get("lora_slot", -1) >= 0 for r in rows)
        graphs = self._store(sampled, lora)
        if Bb not in graphs:
            # capture's warm-up overwrites the shared output buffer, which may hold
            # the in-flight step's tokens that this launch gathers from
            saved = self.out.clone()
            self.capture(Bb, sampled, lora)
            self.out.copy_(saved)
        k = self.slot_k
        self.slot_k ^= 1
        ev = self.staging_ev[k]
        if ev is not None:
            ev.synchronize()
        stg = self.staging[k]
        a = stg.numpy()
        P = self.maxp
        a[self.o_pos:self.o_pos + Bb] = 0
        a[self.o_sl:self.o_sl + Bb] = 0
        a[self.o_src:self.o_src + Bb] = -1
        a[self.o_hid:self.o_hid + Bb] = 0
        slots = a[self.o_slots:self.o_slots + 2 * self.Bmax].view(np.int64)
        slots[:Bb] = -1
        if self.ring:
            rslots = a[self.o_rslots:self.o_rslots + 2 * self.Bmax].view(np.int64)
            rslots[:Bb] = -1
            rpt = a[self.o_rpt:self.o_rpt + self.Bmax * P].reshape(self.Bmax, P)
        if self.rec is not None:
            a[self.o_ss:self.o_ss + Bb] = self.rec.scratch
        a[self.o_lora:self.o_lora + Bb] = -1
        pt = a[self.o_pt:self.o_pt + self.Bmax * P].reshape(self.Bmax, P)
        if sampled:
            keys = a[self.o_key:self.o_key + 2 * self.Bmax].view(np.uint64)
            steps = a[self.o_step:self.o_step + 2 * self.Bmax].view(np.int64)
            temp = a[self.o_temp:self.o_temp + self.Bmax].view(np.float32)
            topk = a[self.o_topk:self.o_topk + self.Bmax]
            topp = a[self.o_topp:self.o_topp + self.Bmax].view(np.float32)
            minp = a[self.o_minp:self.o_minp + self.Bmax].view(np.float32)
            temp[:Bb] = 0.0
        prev_idx = {}
        if chained_from is not None:
            prev_where = chained_from[1][3]
            for j, r in enumerate(chained_from[0].rows):
                prev_idx[id(r.state)] = prev_where[j]
        for i0, r in enumerate(rows):
            i = where[i0]
            st = r.state
            p = r.start
            mm = st.req.mm
            a[self.o_pos + i] = p + (mm["delta"] if mm is not None and p >= mm["prompt_len"] else 0)
            a[self.o_sl + i] = p + 1
            slots[i] = st.seq.slot(p)
            if self.rec is not None:
                a[self.o_ss + i] = st.seq.state_slot
            if lora:
                a[self.o_lora + i] = st.extra.get("lora_slot", -1)
            pg = st.seq.pages
            pt[i, :len(pg)] = pg
            if self.ring:
                rslots[i] = st.seq.ring_slot(p)
                rpt[i] = st.seq.ring_table(P)
            if sampled:
                sp = st.req.sampling
                keys[i] = row_key(st)
                # the Philox counter is the index of the token being drawn: accepted
                # tokens plus the in-flight step's placeholder, as the eager sampler counts
                steps[i] = st.gen_step + (1 if st.all_tokens[-1] == PENDING else 0)
                temp[i] = sp.temperature if not sp.greedy else 0.0
                topk[i] = sp.top_k
                topp[i] = sp.top_p
                minp[i] = sp.min_p
            tok = st.all_tokens[p]
            if tok == PENDING:
                a[self.o_src + i] = prev_idx[id(st)]
            else:
                a[self.o_hid + i] = tok
        nbytes = self.n_i32 * 4
        self.packed.copy_(stg, non_blocking=True)
        self.h2d_bytes += nbytes
        e = torch.cuda.Event()
        e.record()
        self.staging_ev[k] = e
        if self.gather_fn is not None:
            self.gather_fn(self.out, self.src, self.hid, self.ids, Bb)
        else:
            L = _lib.lib()
            _lib.check(L.b200_gather_tokens(self.out.data_ptr(), self.src.data_ptr(), self.hid.data_ptr(),
                                            self.ids.data_ptr(), Bb, _lib.stream_ptr(self.dev)), "gather_tokens")
            _lib.count(1)
        self.model.begin_step()
        graphs[Bb].replay()
        _lib.count(self.launches_per_replay.get(self._key(Bb, sampled, lora), 0))
        ko = self.out_k
        self.out_k = (self.out_k + 1) % len(self.host_out)
        m = max(where) + 1 if where else 0
        self.host_out[ko][:m].copy_(self.out[:m], non_blocking=True)
        self.host_flags[ko][:m].copy_(self.flags[:m], non_blocking=True)
        self.d2h_bytes += 8 * m
        done = torch.cuda.Event()
        done.record()
        return (ko, done, n, where)

    def read_tokens(self, handle, n):
        """(tokens, non-finite flags) of the plan rows of a launched step."""
        ko, done, n0, where = handle
        done.synchronize()
        h = self.host_out[ko].tolist()
        f = self.host_flags[ko].tolist()
        return [h[where[i]] for i in range(n)], [f[where[i]] for i in range(n)]
