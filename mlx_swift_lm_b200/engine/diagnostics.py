"""Engine diagnostics: step profiler, attention-metadata capture and replay,
logit diagnostics, teacher-forced scores.

Parity: the reference's CBv2 diagnostics (CBv2AttentionMetadata*.swift,
CBv2AttentionPacket*.swift, CBv2AttentionReplay*.swift - capture the
attention inputs of a step and replay them; CBv2LogitDiagnostic.swift;
ForwardShapeV2.swift:3 - the engine's ``forward_shapes`` recorder;
CBv2TeacherForcedScores.swift; StepProfilerV2.swift:15, enabled there by
``CBV2_STEP_PROFILE=1`` and here by ``B200LM_STEP_PROFILE=1`` or
``EngineV2.diagnostics = Diagnostics(profile=True)``).

All of it is opt-in and off the hot path: the profiler records one pair of
CUDA events per eager forward and reads them when a summary is requested.
"""
from __future__ import annotations

import math
import os
import statistics
import time
from dataclasses import dataclass, field

import torch

from ..models.batch import ForwardBatch

_META_FIELDS = ("input_ids", "positions", "slots", "dec_page_table", "dec_seq_lens", "pf_cu_q", "pf_pos0",
                "pf_page_table", "logit_idx", "state_slots")


@dataclass
class StepRecord:
    step: int
    rows: int
    decode_rows: int
    tokens: int
    wall_ms: float
    device_ms: float | None = None
    events: tuple | None = None


@dataclass
class LogitReport:
    step: int
    row: int
    top_ids: list
    top_probs: list
    entropy: float
    non_finite: int


@dataclass
class Diagnostics:
    profile: bool = field(default_factory=lambda: os.environ.get("B200LM_STEP_PROFILE", "0") == "1")
    capture_attention: bool = False
    logit_topk: int = 0  # > 0: keep top-k / entropy of every sampled row
    max_records: int = 100000
    steps: list = field(default_factory=list)
    captures: list = field(default_factory=list)
    logits: list = field(default_factory=list)

    # ------------------------------------------------------------------ hooks
    def begin_forward(self, device):
        if not self.profile:
            return None
        t0 = time.perf_counter()
        ev = None
        if device.type == "cuda":
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        return t0, ev

    def end_forward(self, token, step: int, fb: ForwardBatch, logits: torch.Tensor | None):
        if token is not None:
            t0, ev = token
            if ev is not None:
                ev[1].record()
            if len(self.steps) < self.max_records:
                self.steps.append(StepRecord(step, _rows(fb), fb.num_decode, fb.num_tokens,
                                             (time.perf_counter() - t0) * 1e3, None, ev))
        if self.capture_attention and len(self.captures) < self.max_records:
            self.captures.append(capture_metadata(fb))
        if self.logit_topk > 0 and logits is not None and len(self.logits) < self.max_records:
            self.logits.extend(logit_report(step, logits, self.logit_topk))

    # ------------------------------------------------------------------ summaries
    def step_summary(self) -> dict:
        """p50 / p90 / max of the wall and device times of profiled forwards."""
        for r in self.steps:
            if r.events is not None and r.device_ms is None:
                r.events[1].synchronize()
                r.device_ms = r.events[0].elapsed_time(r.events[1])
                r.events = None
        out = {"forwards": len(self.steps)}
        for key in ("wall_ms", "device_ms"):
            v = sorted(getattr(r, key) for r in self.steps if getattr(r, key) is not None)
            if v:
                out[key] = {"p50": statistics.median(v), "p90": v[min(len(v) - 1, int(0.9 * len(v)))], "max": v[-1]}
        out["tokens"] = sum(r.tokens for r in self.steps)
        return out


def _rows(fb: ForwardBatch) -> int:
    return fb.num_decode + len(fb.pf_cu_q_host or [0]) - 1


def capture_metadata(fb: ForwardBatch) -> dict:
    """Host copy of a forward batch's attention inputs (positions, K/V slots,
    page tables, sequence lengths, chunk offsets): enough to replay it."""
    d = {"num_decode": fb.num_decode, "dec_max_parts": fb.dec_max_parts, "pf_cu_q_host": fb.pf_cu_q_host,
         "logit_idx_host": fb.logit_idx_host, "row_ranks": fb.row_ranks}
    for n in _META_FIELDS:
        t = getattr(fb, n)
        d[n] = None if t is None else t.detach().cpu().clone()
    return d


def replay_batch(meta: dict, device) -> ForwardBatch:
    """The captured forward batch, rebuilt on `device`."""
    kw = {n: (None if meta[n] is None else meta[n].to(device)) for n in _META_FIELDS}
    fb = ForwardBatch(input_ids=kw.pop("input_ids"), positions=kw.pop("positions"), slots=kw.pop("slots"),
                      num_decode=meta["num_decode"], dec_max_parts=meta["dec_max_parts"])
    for n, v in kw.items():
        setattr(fb, n, v)
    fb.pf_cu_q_host, fb.logit_idx_host, fb.row_ranks = meta["pf_cu_q_host"], meta["logit_idx_host"], meta["row_ranks"]
    return fb


def logit_report(step: int, logits: torch.Tensor, k: int) -> list[LogitReport]:
    """Top-k probabilities, entropy and the count of non-finite logits of
    every row."""
    lg = logits.float()
    bad = (~torch.isfinite(lg)).sum(-1)
    p = torch.softmax(torch.nan_to_num(lg, nan=-math.inf), -1)
    ent = -(p * torch.log(p.clamp(min=1e-30))).sum(-1)
    tp, ti = torch.topk(p, min(k, p.shape[-1]), -1)
    tp, ti, ent, bad = tp.cpu(), ti.cpu(), ent.cpu(), bad.cpu()
    return [LogitReport(step, i, ti[i].tolist(), tp[i].tolist(), float(ent[i]), int(bad[i]))
            for i in range(lg.shape[0])]


@torch.no_grad()
def teacher_forced_scores(engine, prompt: list[int], continuation: list[int]) -> list[float]:
    """Log-probability of each continuation token given the prompt and the
    preceding continuation tokens (one prefill over prompt + continuation)."""
    from ..kv.paged import SequenceKV

    toks = list(prompt) + list(continuation)
    seq = SequenceKV(engine.kv)
    try:
        if not seq.ensure(len(toks)):
            raise RuntimeError("no KV capacity")
        dev = engine.device
        i32 = dict(dtype=torch.int32)
        fb = ForwardBatch(input_ids=torch.tensor(toks, **i32).to(dev),
                          positions=torch.arange(len(toks), **i32).to(dev),
                          slots=torch.tensor(seq.slots(0, len(toks)), dtype=torch.int64).to(dev), num_decode=0,
                          pf_cu_q=torch.tensor([0, len(toks)], **i32).to(dev), pf_cu_q_host=[0, len(toks)],
                          pf_pos0=torch.tensor([0], **i32).to(dev),
                          pf_page_table=torch.tensor([seq.pages], **i32).to(dev))
        if engine.kv.rec is not None:
            fb.state_slots = torch.tensor([seq.state_slot], **i32).to(dev)
        n0 = len(prompt)
        fb.logit_idx_host = list(range(n0 - 1, len(toks) - 1))
        fb.logit_idx = torch.tensor(fb.logit_idx_host, dtype=torch.int64).to(dev)
        logits = engine.model.forward(fb, engine.kv).float()
        lp = torch.log_softmax(logits, -1)
        tgt = torch.tensor(continuation, dtype=torch.int64, device=lp.device)
        return lp.gather(1, tgt[:, None])[:, 0].tolist()
    finally:
        seq.release()


def timeline_summary(marks, title: str = "") -> str:
    """Text summary of device timeline marks (``ops._lib.timeline_read``):
    each kernel's cost in the dependent chain is the time from its mark to the
    next kernel's (its predecessor finished at its mark, it finished at the
    next). Tagged points inside kernels (collective waits returning, signals
    going out) are listed in place. Totals per launch signature follow."""
    lines = [title] if title else []
    kern = [m for m in marks if not isinstance(m[1], int)]
    if len(kern) < 2:
        return "\n".join(lines + ["(fewer than two kernel marks)"])
    t0 = marks[0][0]
    agg: dict = {}
    ki = 0
    for t, sig in marks:
        if isinstance(sig, int):
            lines.append(f"{(t - t0) / 1e3:10.2f} us      -     tag 0x{sig:x}")
            continue
        if ki + 1 >= len(kern):
            break
        dt = (kern[ki + 1][0] - t) / 1e3
        ki += 1
        lines.append(f"{(t - t0) / 1e3:10.2f} us  {dt:8.2f} us  grid {sig[0]}x{sig[1]}x{sig[2]} block {sig[3]}")
        a = agg.setdefault(sig, [0, 0.0])
        a[0] += 1
        a[1] += dt
    total = (kern[-1][0] - kern[0][0]) / 1e3
    lines.append(f"span {total:.2f} us over {len(kern)} kernel marks; per signature (count, total us, mean us, share):")
    for sig, (n, tot) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        lines.append(f"  grid {sig[0]}x{sig[1]}x{sig[2]} block {sig[3]:4d}: {n:5d} {tot:10.2f} {tot / n:8.2f} "
                     f"{tot / total:6.1%}")
    return "\n".join(lines)
