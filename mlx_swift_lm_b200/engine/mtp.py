"""MTP speculative decoding inside the continuous-batching engine.

Parity: the CBv2 MTP round (MTP/EngineLoopV2+MTP.swift:15, planning
+MTPPlanning.swift, drafting CBv2MTPRoundDriver.swift:52-80, one rectangular
target verify +MTPTargetVerification.swift, accept walk and per-row rollback
+MTPFinalize.swift:101, PagedSequenceKV.swift:412) for greedy rows.

One round for the decode rows of a step, each with pending token x at
position p (sampled, no K/V yet) and MTP K/V valid below position m:

1. draft step 1: the MTP module runs over positions m..p of every row as one
   chunk, with the target's hiddens h_{m-1}..h_{p-1} (kept from the previous
   verify), writing exact MTP K/V for them; its output at p drafts d_1.
2. draft steps 2..k: one position each (p+1 .. p+k-1), fed the drafted token
   and the module's own output hidden (speculative MTP K/V).
3. verify: one target forward over [x, d_1 .. d_k] at p..p+k for every row
   (a (k+1)-token chunk per row), returning logits and hiddens.
4. accept: greedy: a = leading matches of d_{j+1} with the target's argmax at
   column j; emit d_1..d_a and the target's token at column a. The target K/V
   of positions p+a+1.. is rolled back (seq length p+a+1); MTP K/V keeps only
   the exact step-1 positions (up to p). The verify hiddens of columns 0..a
   become the next round's step-1 inputs.

`acceptance="bernoulli"` replaces the match test with a seeded Bernoulli(p)
schedule (a = leading successes, capped at k), for throughput measurement on
random weights where drafts never match; emitted tokens are then the drafts.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .. import ops
from ..kv.paged import SequenceKV
from ..models.batch import ForwardBatch
from ..ops.attention import decode_max_parts


@dataclass
class MTPConfig:
    k: int = 3  # draft depth (the maximum depth when adaptive)
    acceptance: str = "exact"  # exact | bernoulli
    p: float = 0.7
    seed: int = 0
    adaptive: bool = False  # choose the depth per round (engine.mtp_depth.DepthController)
    max_rows: int = 0  # > 0: steps with more decode rows run without drafts (bounded drafter work)
    graph_round: bool = True  # fixed-geometry rounds (engine.mtp_graph), CUDA graphs on GPU


@dataclass
class MTPStats:
    rounds: int = 0
    rows: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0


class MTPDriver:
    def __init__(self, engine, module, config: MTPConfig | None = None):
        self.eng = engine
        self.mod = module
        self.cfg = config or MTPConfig()
        # the MTP history of a row never exceeds its target history
        self.kv = module.new_kv(max_tokens=(engine.kv.num_pages - 1) * 16, kv_fp8=engine.cfg.kv_fp8)
        self.rng = np.random.default_rng(self.cfg.seed)
        self.stats = MTPStats()
        self.depth = None
        if self.cfg.adaptive:
            from .mtp_depth import DepthController

            self.depth = DepthController(self.cfg.k)
        self._h2d = 0  # step inputs copied host -> device (eager rounds)
        self._d2h = 0  # drafts + target tokens read back (eager rounds)
        self.runner = None
        m = engine.model
        if (self.cfg.graph_round and m.tp.world == 1 and getattr(m, "pp_stages", 1) == 1
                and getattr(m, "dp_world", 1) == 1):
            from .mtp_graph import MTPGraphRunner

            self.runner = MTPGraphRunner(self)

    @property
    def h2d_bytes(self):
        return self._h2d + (self.runner.h2d_bytes if self.runner is not None else 0)

    @h2d_bytes.setter
    def h2d_bytes(self, v):
        self._h2d = v - (self.runner.h2d_bytes if self.runner is not None else 0)

    @property
    def d2h_bytes(self):
        return self._d2h + (self.runner.d2h_bytes if self.runner is not None else 0)

    @d2h_bytes.setter
    def d2h_bytes(self, v):
        self._d2h = v - (self.runner.d2h_bytes if self.runner is not None else 0)

    # ------------------------------------------------------------------ row state
    def on_first_token(self, st, hidden_row: torch.Tensor):
        """A row just sampled its first token: MTP history starts at its position."""
        self.drop(st)
        st.extra["mtp_seq"] = SequenceKV(self.kv)
        st.extra["mtp_p0"] = len(st.all_tokens) - 1  # position of the pending token
        st.extra["mtp_m"] = st.extra["mtp_p0"]
        st.extra["mtp_h"] = hidden_row.reshape(1, -1)
        if self.runner is not None and not self.runner.attach(st, hidden_row):
            self.drop(st)

    def drop(self, st):
        seq = st.extra.pop("mtp_seq", None)
        if seq is not None:
            seq.release()
        if self.runner is not None:
            self.runner.detach(st)
        for k in ("mtp_p0", "mtp_m", "mtp_h"):
            st.extra.pop(k, None)

    def eligible(self, plan) -> bool:
        if not plan.pure_decode:
            return False
        if self.cfg.max_rows > 0 and len(plan.rows) > self.cfg.max_rows:
            return False
        for r in plan.rows:
            st = r.state
            sp = st.req.sampling
            if (not sp.greedy or st.req.token_constraint is not None or sp.logprobs or sp.top_logprobs > 0
                    or sp.needs_processing or "mtp_h" not in st.extra or st.req.mm is not None
                    or "budget" in st.extra):
                return False
        return True

    # ------------------------------------------------------------------ round
    def _ensure(self, rows, k: int | None = None) -> bool:
        k = self.cfg.k if k is None else k
        for r in rows:
            st = r.state
            if not self.eng.sched._ensure(st, r.start + k + 1):
                return False
            local_end = r.start + k - st.extra["mtp_p0"]
            if not st.extra["mtp_seq"].ensure(local_end):
                return False
        return True

    def _to_dev(self, fb: ForwardBatch):
        dev = self.eng.device
        if dev.type == "cuda":
            for name in ("input_ids", "positions", "slots", "dec_page_table", "dec_seq_lens", "pf_cu_q", "pf_pos0",
                         "pf_page_table", "logit_idx"):
                t = getattr(fb, name)
                if t is not None and not t.is_cuda:
                    self.h2d_bytes += t.numel() * t.element_size()
                    setattr(fb, name, t.pin_memory().to(dev, non_blocking=True))
        return fb

    def _chunk_batch(self, toks, pos0, lens, seqs, local0, logit_last=True) -> ForwardBatch:
        """Rows as prefill chunks: row i covers positions pos0[i] .. +lens[i]-1
        stored at local K/V indices local0[i] .. of seqs[i]."""
        ids, pos, slots, cu, p0 = [], [], [], [0], []
        maxp = max(len(s.pages) for s in seqs)
        pt = np.zeros((len(seqs), maxp), np.int32)
        for i, s in enumerate(seqs):
            n = lens[i]
            ids.extend(toks[i])
            pos.extend(range(pos0[i], pos0[i] + n))
            slots.extend(s.slots(local0[i], n))
            cu.append(cu[-1] + n)
            p0.append(local0[i])
            pt[i, :len(s.pages)] = s.pages
        fb = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.int32), positions=torch.tensor(pos, dtype=torch.int32),
                          slots=torch.tensor(slots, dtype=torch.int64), num_decode=0)
        fb.pf_cu_q = torch.tensor(cu, dtype=torch.int32)
        fb.pf_cu_q_host = cu
        fb.pf_pos0 = torch.tensor(p0, dtype=torch.int32)
        fb.pf_page_table = torch.from_numpy(pt)
        if logit_last:
            fb.logit_idx = torch.tensor([c - 1 for c in cu[1:]], dtype=torch.int64)
        return fb

    def _decode_batch(self, toks_dev, positions, seqs, local) -> ForwardBatch:
        B = len(seqs)
        maxp = max(len(s.pages) for s in seqs)
        pt = np.zeros((B, maxp), np.int32)
        for i, s in enumerate(seqs):
            pt[i, :len(s.pages)] = s.pages
        sl = np.array([l + 1 for l in local], np.int32)
        fb = ForwardBatch(input_ids=toks_dev, positions=torch.tensor(positions, dtype=torch.int32),
                          slots=torch.tensor([s.slot(l) for s, l in zip(seqs, local)], dtype=torch.int64),
                          num_decode=B, dec_page_table=torch.from_numpy(pt), dec_seq_lens=torch.from_numpy(sl),
                          dec_max_parts=decode_max_parts(int(sl.max())))
        return self._to_dev(fb)

    def round(self, plan):
        """Run one MTP round for a pure-decode greedy plan. Returns the emitted
        events, or None when KV capacity does not allow a round (the caller
        then runs a normal decode step)."""
        import time

        eng = self.eng
        k = self.depth.choose() if self.depth is not None else self.cfg.k
        t_round = time.perf_counter()
        rows = plan.rows
        if not self._ensure(rows, k):
            return None
        if self.runner is not None and self.runner.can_run(plan, k):
            return self._round_fixed(plan, k, t_round)
        return self._round_eager(plan, k, t_round)

    def _draw_accepts(self, n: int, k: int) -> list[int]:
        out = []
        for _ in range(n):
            a = 0
            while a < k and self.rng.random() < self.cfg.p:
                a += 1
            out.append(a)
        return out

    def _round_fixed(self, plan, k: int, t_round: float):
        """A round through the fixed-geometry runner (one graph replay)."""
        import time

        eng = self.eng
        rows = plan.rows
        forced = self._draw_accepts(len(rows), k) if self.cfg.acceptance == "bernoulli" else None
        emit, acc = self.runner.run(plan, k, forced)
        V = eng.model.cfg.vocab_size
        for i in range(len(rows)):
            a = int(acc[i])
            if not (0 <= a <= k) or any(not (0 <= int(t) < V) for t in emit[i, :a + 1]):
                raise RuntimeError(f"MTP round returned accept count {a} / tokens {emit[i].tolist()} for row {i}")
        events = []
        st_ = self.stats
        st_.rounds += 1
        st_.rows += len(rows)
        acc_rows = []
        for i, r in enumerate(rows):
            st = r.state
            p = r.start
            a = int(acc[i])
            st_.drafted += k
            st_.accepted += a
            acc_rows.append(a)
            st.extra["mtp_seq"].num_tokens = p + 1 - st.extra["mtp_p0"]
            st.seq.num_tokens = p + a + 1
            st.extra["mtp_m"] = p + 1
            for t in emit[i, :a + 1]:
                st_.emitted += 1
                events += eng._accept_token(st, int(t), None)
                if st.status.name == "FINISHED":
                    break
        if self.depth is not None:
            self.depth.observe(k, acc_rows, time.perf_counter() - t_round)
        return events

    def _round_eager(self, plan, k: int, t_round: float):
        import time

        eng = self.eng
        rows = plan.rows
        states = [r.state for r in rows]
        B = len(rows)
        p = [r.start for r in rows]
        mseqs = [st.extra["mtp_seq"] for st in states]
        p0 = [st.extra["mtp_p0"] for st in states]
        # ---- draft step 1: positions m..p per row, exact hiddens
        m = [st.extra["mtp_m"] for st in states]
        lens = [p[i] - m[i] + 1 for i in range(B)]
        toks = [states[i].all_tokens[m[i]:p[i] + 1] for i in range(B)]
        hid = torch.cat([st.extra["mtp_h"] for st in states], 0)
        assert hid.shape[0] == sum(lens), "MTP hidden history out of step with the token history"
        fb = self._to_dev(self._chunk_batch(toks, m, lens, mseqs, [m[i] - p0[i] for i in range(B)]))
        logits, h = self.mod.forward(fb, self.kv, hid)
        for i in range(B):
            mseqs[i].num_tokens = p[i] + 1 - p0[i]
        d = ops.argmax(logits)
        drafts = [d]
        # ---- draft steps 2..k (speculative MTP K/V)
        for j in range(1, k):
            fbd = self._decode_batch(d, [p[i] + j for i in range(B)], mseqs, [p[i] + j - p0[i] for i in range(B)])
            logits, h = self.mod.forward(fbd, self.kv, h)
            d = ops.argmax(logits)
            drafts.append(d)
        D = torch.stack(drafts, 1)  # [B, k] int32
        # ---- verify: [x, d_1..d_k] at p..p+k
        x = torch.tensor([states[i].all_tokens[p[i]] for i in range(B)], dtype=torch.int32, device=D.device)
        vt = torch.cat([x[:, None], D], 1)  # [B, k+1]
        seqs = [st.seq for st in states]
        fbv = self._chunk_batch([[0] * (k + 1)] * B, p, [k + 1] * B, seqs, p, logit_last=False)
        fbv.input_ids = vt.reshape(-1)
        fbv.row_ranks = eng._row_ranks(rows)
        fbv = self._to_dev(fbv)
        pred, vh = eng.model.forward_greedy_both(fbv, eng.kv)
        pred = pred.view(B, k + 1)
        both = torch.cat([pred, D], 1).cpu().numpy()
        self.d2h_bytes += both.nbytes
        pred_h, D_h = both[:, :k + 1], both[:, k + 1:]
        vh = vh.view(B, k + 1, -1)
        events = []
        st_ = self.stats
        st_.rounds += 1
        st_.rows += B
        acc_rows = []
        for i, st in enumerate(states):
            if self.cfg.acceptance == "bernoulli":
                a = self._draw_accepts(1, k)[0]
            else:
                a = 0
                while a < k and D_h[i, a] == pred_h[i, a]:
                    a += 1
            emit = [int(t) for t in D_h[i, :a]] + [int(pred_h[i, a])]
            st_.drafted += k
            st_.accepted += a
            acc_rows.append(a)
            # target K/V: x and the accepted drafts; the rest is rolled back
            st.seq.num_tokens = p[i] + a + 1
            # next round: step-1 history p+1 .. p+a+1 with verify hiddens of columns 0..a
            st.extra["mtp_m"] = p[i] + 1
            st.extra["mtp_h"] = vh[i, :a + 1].contiguous()
            for t in emit:
                st_.emitted += 1
                events += eng._accept_token(st, t, None)
                if st.status.name == "FINISHED":
                    break
        if self.depth is not None:
            # the round ends with the host readback above: its wall time is the round's cost
            self.depth.observe(k, acc_rows, time.perf_counter() - t_round)
        return events
