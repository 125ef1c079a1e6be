"""MTP rounds with a fixed launch geometry, captured as one CUDA graph per
(batch bucket, draft depth).

The eager round (:mod:`.mtp`) runs the first draft step as prefill chunks
of varying length (the positions each row accepted last round), which no
captured graph can replay. Here every forward of the round is a batch of
decode rows:

* draft step 1: a window of k + 1 rows per request at positions p-k .. p.
  The positions m .. p the request has not fed to the draft module yet are
  right-aligned in the window and write exact draft K/V; the rows before m
  are inert (no K/V write, a one-key context) and their outputs unused. The
  target hiddens they consume sit right-aligned in a per-request history row
  on the device (``hist [slots, k+1, H]``), written by the previous round's
  accept kernel.
* draft steps 2 .. k: one row per request fed the previous draft token and
  the module's own hidden (speculative draft K/V).
* verify: k + 1 decode rows per request at p .. p+k over [x, d_1 .. d_k],
  each attending causally to its own prefix. Decode rows use the decode
  kernels and launch geometry, so the verify computes exactly what plain
  decode steps compute: the emitted tokens are those of non-speculative
  greedy decoding.
* accept (``csrc/kernels/mtp.cu``): the greedy accept walk, the emitted
  tokens, and the history rows of the next round, on the device.

The host packs one input buffer per round (one copy), replays the graph and
reads back the emitted tokens and accept counts (one copy): the round
structure of the reference (MTP/EngineLoopV2+MTP.swift:15,
CBv2MTPRoundDriver.swift:52-80, +MTPTargetVerification.swift,
+MTPFinalize.swift:101) with its launches recorded once.
On CPU the same body runs eagerly (tests compare it with the eager round).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..models.batch import ForwardBatch
from ..ops import _lib
from ..ops.attention import SCRATCH, decode_max_parts, merge_counters


class _Round:
    """Device buffers and (on CUDA) the captured graph of one (B, k)."""

    def __init__(self, runner, B: int, k: int):
        self.B, self.k = B, k
        T1, P, dev = B * (k + 1), runner.P, runner.dev
        self.T1 = T1
        o = {}
        n = 0

        def take(name, count, wide=False):
            nonlocal n
            if wide:
                n += n % 2
            o[name] = n
            n += count * (2 if wide else 1)

        take("s1_ids", T1)
        take("s1_pos", T1)
        take("s1_sl", T1)
        take("s1_pt", T1 * P)
        take("hs", B)
        take("dr_pos", max(k - 1, 1) * B)
        take("dr_sl", max(k - 1, 1) * B)
        take("dr_pt", B * P)
        take("x", B)
        take("v_pos", T1)
        take("v_sl", T1)
        take("v_pt", T1 * P)
        take("forced", B)
        take("s1_slots", T1, wide=True)
        take("dr_slots", max(k - 1, 1) * B, wide=True)
        take("v_slots", T1, wide=True)
        self.off, self.n = o, n
        self.packed = torch.zeros(n, dtype=torch.int32, device=dev)
        self.staging = torch.zeros(n, dtype=torch.int32)
        if dev.type == "cuda":
            self.staging = self.staging.pin_memory()
        self.copy_ev = None

        def v(name, count, shape=None, wide=False):
            t = self.packed[o[name]:o[name] + count * (2 if wide else 1)]
            if wide:
                t = t.view(torch.int64)
            return t.view(*shape) if shape else t

        self.s1_ids, self.s1_pos, self.s1_sl = v("s1_ids", T1), v("s1_pos", T1), v("s1_sl", T1)
        self.s1_pt = v("s1_pt", T1 * P, (T1, P))
        self.s1_slots = v("s1_slots", T1, wide=True)
        self.hs = v("hs", B)
        nd = max(k - 1, 1)
        self.dr_pos, self.dr_sl = v("dr_pos", nd * B, (nd, B)), v("dr_sl", nd * B, (nd, B))
        self.dr_slots = v("dr_slots", nd * B, (nd, B), wide=True)
        self.dr_pt = v("dr_pt", B * P, (B, P))
        self.x = v("x", B)
        self.v_pos, self.v_sl = v("v_pos", T1), v("v_sl", T1)
        self.v_pt = v("v_pt", T1 * P, (T1, P))
        self.v_slots = v("v_slots", T1, wide=True)
        self.forced = v("forced", B)
        self.last = (torch.arange(B, device=dev, dtype=torch.int64) * (k + 1) + k)
        self.D = torch.zeros(B, k, dtype=torch.int32, device=dev)
        self.vt = torch.zeros(T1, dtype=torch.int32, device=dev)
        self.res = torch.zeros(B, k + 2, dtype=torch.int32, device=dev)  # emit [k+1] | a
        self.host_res = torch.zeros(B, k + 2, dtype=torch.int32)
        if dev.type == "cuda":
            self.host_res = self.host_res.pin_memory()
        self.graph = None
        self.launches = 0


class MTPGraphRunner:
    def __init__(self, driver):
        eng = driver.eng
        self.drv, self.eng, self.mod = driver, eng, driver.mod
        self.dev = eng.device
        self.P = eng.max_pages
        self.max_parts = decode_max_parts(eng.cfg.max_model_len)
        mc = eng.cfg.scheduler.max_concurrent_requests
        self.buckets = sorted({b for b in eng.cfg.graph_buckets if b <= mc} | {mc})
        m = eng.model
        self.Hd = m.cfg.hidden_size
        # history rows: one per running request plus a scratch row for bucket padding
        self.S = mc + 1
        self.pad_slot = self.S - 1
        self.hist = torch.zeros(self.S, driver.cfg.k + 1, self.Hd, dtype=m.dtype, device=self.dev)
        self.free = list(range(self.S - 1))
        self.rounds: dict[tuple[int, int], _Round] = {}
        self.pool = None
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.use_graphs = self.dev.type == "cuda" and eng.cfg.use_cuda_graphs
        if self.dev.type == "cuda":
            # decode scratch for the widest batch of the round (k+1 rows per request), before any
            # capture: a later growth would move buffers that captured graphs point to
            T1 = self.buckets[-1] * (driver.cfg.k + 1)
            for mdl in (m, self.mod.inner):
                H, D = mdl.attn_scratch_dims()
                SCRATCH.get(self.dev, "dec_acc", T1 * H * self.max_parts * D)
                SCRATCH.get(self.dev, "dec_ml", T1 * H * self.max_parts * 2)
                merge_counters(self.dev, T1 * max(mdl.KVH, 1))
            ops.WORKSPACE.reserve(self.dev, 512 << 20)
            if eng.graphs is not None:
                eng.graphs.invalidate()

    # ------------------------------------------------------------------ row state
    def attach(self, st, hidden_row: torch.Tensor):
        """A request enters MTP decoding with the target hidden of its last prompt position."""
        if "mtp_hslot" not in st.extra:
            if not self.free:
                return False
            st.extra["mtp_hslot"] = self.free.pop()
        k = self.drv.cfg.k
        self.hist[st.extra["mtp_hslot"], k] = hidden_row.reshape(-1).to(self.hist.dtype)
        return True

    def detach(self, st):
        s = st.extra.pop("mtp_hslot", None)
        if s is not None:
            self.free.append(s)

    def can_run(self, plan, k: int) -> bool:
        return (k <= self.drv.cfg.k and len(plan.rows) <= self.buckets[-1]
                and all("mtp_hslot" in r.state.extra for r in plan.rows))

    # ------------------------------------------------------------------ round
    def _bucket(self, n):
        for b in self.buckets:
            if b >= n:
                return b
        return None

    def _fb(self, R: _Round, stage: str, j: int = 0) -> ForwardBatch:
        mp = self.max_parts
        if stage == "s1":
            return ForwardBatch(input_ids=R.s1_ids, positions=R.s1_pos, slots=R.s1_slots, num_decode=R.T1,
                                dec_page_table=R.s1_pt, dec_seq_lens=R.s1_sl, dec_max_parts=mp, logit_idx=R.last)
        if stage == "dr":
            return ForwardBatch(input_ids=None, positions=R.dr_pos[j], slots=R.dr_slots[j], num_decode=R.B,
                                dec_page_table=R.dr_pt, dec_seq_lens=R.dr_sl[j], dec_max_parts=mp)
        return ForwardBatch(input_ids=R.vt, positions=R.v_pos, slots=R.v_slots, num_decode=R.T1,
                            dec_page_table=R.v_pt, dec_seq_lens=R.v_sl, dec_max_parts=mp)

    def _body(self, R: _Round):
        B, k = R.B, R.k
        mkv = self.drv.kv
        K = self.drv.cfg.k
        h_in = self.hist.index_select(0, R.hs.long())[:, K - k:].reshape(R.T1, self.Hd)
        logits, h = self.mod.forward(self._fb(R, "s1"), mkv, h_in)
        d = ops.argmax(logits)
        R.D[:, 0].copy_(d)
        for j in range(1, k):
            fb = self._fb(R, "dr", j - 1)
            fb.input_ids = d
            logits, h = self.mod.forward(fb, mkv, h)
            d = ops.argmax(logits)
            R.D[:, j].copy_(d)
        vt = R.vt.view(B, k + 1)
        vt[:, 0].copy_(R.x)
        vt[:, 1:].copy_(R.D)
        logits, vh = self.eng.model.forward(self._fb(R, "v"), self.eng.kv, return_both=True)
        pred = ops.argmax(logits)
        self._accept(R, pred, vh)

    def _accept(self, R: _Round, pred, vh):
        B, k = R.B, R.k
        emit, acc = R.res[:, :k + 1], R.res[:, k + 1]
        if R.packed.is_cuda:
            # res rows: k + 1 emitted tokens, then the accept count (one contiguous [B, k+2] buffer)
            assert R.res.is_contiguous() and R.D.is_contiguous() and pred.is_contiguous() and vh.is_contiguous()
            rc = _lib.lib().b200_mtp_accept(pred.data_ptr(), R.D.data_ptr(), R.forced.data_ptr(), k,
                                            R.hs.data_ptr(), self.S, self.drv.cfg.k, vh.data_ptr(), self.Hd,
                                            self.hist.data_ptr(), R.res.data_ptr(), B, _lib.stream_ptr(self.dev))
            _lib.check(rc, "mtp_accept")
            _lib.count(1)
            return
        P = pred.view(B, k + 1)
        vh = vh.view(B, k + 1, -1)
        for r in range(B):
            f = int(R.forced[r])
            if f >= 0:
                a = min(f, k)
            else:
                a = 0
                while a < k and int(R.D[r, a]) == int(P[r, a]):
                    a += 1
            row = [int(t) for t in R.D[r, :a]] + [int(P[r, a])] + [-1] * (k - a)
            emit[r] = torch.tensor(row, dtype=torch.int32)
            acc[r] = a
            K = self.drv.cfg.k
            self.hist[int(R.hs[r]), K - a:] = vh[r, :a + 1].to(self.hist.dtype)

    def _get(self, B, k) -> _Round:
        R = self.rounds.get((B, k))
        if R is None:
            R = self.rounds[(B, k)] = _Round(self, B, k)
        return R

    def _capture(self, R: _Round):
        m = self.eng.model
        cur = torch.cuda.current_stream(self.dev)
        # warm-up on inert inputs: no K/V writes, one-key contexts, the padding history row
        R.packed.zero_()
        R.s1_slots.fill_(-1)
        R.dr_slots.fill_(-1)
        R.v_slots.fill_(-1)
        R.s1_sl.fill_(1)
        R.dr_sl.fill_(1)
        R.v_sl.fill_(1)
        R.forced.fill_(0)
        R.hs.fill_(self.pad_slot)
        saved = self.hist.clone()
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            for _ in range(2):
                m.begin_step()
                self._body(R)
        cur.wait_stream(s)
        torch.cuda.synchronize(self.dev)
        n0 = _lib.launch_counter[0]
        g = torch.cuda.CUDAGraph()
        m.begin_step()
        with torch.cuda.graph(g, pool=self.pool):
            self._body(R)
        R.launches = _lib.launch_counter[0] - n0
        if self.pool is None:
            self.pool = g.pool()
        R.graph = g
        torch.cuda.synchronize(self.dev)
        self.hist.copy_(saved)

    def run(self, plan, k: int, forced: list[int] | None):
        """One round for the plan's rows; returns (emit [rows, k+1], accepted [rows]) on the host."""
        drv = self.drv
        rows = plan.rows
        n = len(rows)
        B = self._bucket(n)
        R = self._get(B, k)
        if self.use_graphs and R.graph is None:
            self._capture(R)
        if R.copy_ev is not None:
            R.copy_ev.synchronize()
        a = R.staging.numpy()
        o, P, T1 = R.off, self.P, R.T1
        a[:] = 0
        s1_slots = a[o["s1_slots"]:o["s1_slots"] + 2 * T1].view(np.int64)
        dr_slots = a[o["dr_slots"]:o["dr_slots"] + 2 * max(k - 1, 1) * B].view(np.int64).reshape(max(k - 1, 1), B)
        v_slots = a[o["v_slots"]:o["v_slots"] + 2 * T1].view(np.int64)
        s1_slots[:] = -1
        dr_slots[:] = -1
        v_slots[:] = -1
        a[o["s1_sl"]:o["s1_sl"] + T1] = 1
        a[o["dr_sl"]:o["dr_sl"] + max(k - 1, 1) * B] = 1
        a[o["v_sl"]:o["v_sl"] + T1] = 1
        a[o["hs"]:o["hs"] + B] = self.pad_slot
        a[o["forced"]:o["forced"] + B] = -1
        s1_pt = a[o["s1_pt"]:o["s1_pt"] + T1 * P].reshape(T1, P)
        v_pt = a[o["v_pt"]:o["v_pt"] + T1 * P].reshape(T1, P)
        dr_pt = a[o["dr_pt"]:o["dr_pt"] + B * P].reshape(B, P)
        dr_pos = a[o["dr_pos"]:o["dr_pos"] + max(k - 1, 1) * B].reshape(max(k - 1, 1), B)
        dr_sl = a[o["dr_sl"]:o["dr_sl"] + max(k - 1, 1) * B].reshape(max(k - 1, 1), B)
        for i, r in enumerate(rows):
            st = r.state
            p = r.start
            p0, m = st.extra["mtp_p0"], st.extra["mtp_m"]
            mseq, seq = st.extra["mtp_seq"], st.seq
            toks = st.all_tokens
            mp, tp = mseq.pages, seq.pages
            for j in range(k + 1):
                row = i * (k + 1) + j
                w = p - k + j
                a[o["s1_pos"] + row] = max(w, 0)
                s1_pt[row, :len(mp)] = mp
                if w >= m:  # a position the draft module has not seen: exact draft K/V
                    a[o["s1_ids"] + row] = toks[w]
                    s1_slots[row] = mseq.slot(w - p0)
                    a[o["s1_sl"] + row] = w - p0 + 1
                # verify row j: token (x or d_j) at p + j over the target's prefix
                a[o["v_pos"] + row] = p + j
                v_slots[row] = seq.slot(p + j)
                a[o["v_sl"] + row] = p + j + 1
                v_pt[row, :len(tp)] = tp
            for j in range(1, k):
                dr_pos[j - 1, i] = p + j
                dr_slots[j - 1, i] = mseq.slot(p + j - p0)
                dr_sl[j - 1, i] = p + j - p0 + 1
            dr_pt[i, :len(mp)] = mp
            a[o["x"] + i] = toks[p]
            a[o["hs"] + i] = st.extra["mtp_hslot"]
            if forced is not None:
                a[o["forced"] + i] = forced[i]
        R.packed.copy_(R.staging, non_blocking=True)
        self.h2d_bytes += R.n * 4
        if R.packed.is_cuda:
            R.copy_ev = torch.cuda.Event()
            R.copy_ev.record()
        if R.graph is not None:
            self.eng.model.begin_step()
            R.graph.replay()
            _lib.count(R.launches)
        else:
            self._body(R)
        R.host_res.copy_(R.res, non_blocking=True)
        if R.packed.is_cuda:
            torch.cuda.current_stream(self.dev).synchronize()
        self.d2h_bytes += n * (k + 2) * 4
        res = R.host_res[:n].numpy()
        return res[:, :k + 1], res[:, k + 1]
