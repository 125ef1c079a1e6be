"""Batched sampler: per-request parameters vectorised into per-row tensors.

Pipeline order and semantics follow the reference's DefaultSamplerV2
(ContinuousBatchingV2/DefaultSamplerV2.swift:84-183) and LogitsPipelineV2
(LogitsPipelineV2.swift:39-618): raw logprobs first, then logit bias,
penalties, token constraints, temperature / top-k / top-p / min-p, draw.
An all-greedy batch takes the argmax fast path. The RNG key of a row is
(seed mixed with request id) and its counter the row's generation step, so
sampling is reproducible and independent of batch-mates.

CUDA rows run the fused kernels of ``csrc/kernels/sampling.cu``; CPU rows run
the oracle in :mod:`mlx_swift_lm_b200.ops.reference`.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..ops import reference as ref
from .types import TokenLogprob

DEFAULT_SEED = 0x5EED


def row_key(st) -> int:
    sp = st.req.sampling
    seed = sp.seed if sp.seed is not None else DEFAULT_SEED
    return ref.mix_key(int(seed), int(st.req.id))


class Sampler:
    def __init__(self, vocab_size: int, device):
        self.V = vocab_size
        self.device = torch.device(device)

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _penalty_lists(st):
        sp = st.req.sampling
        rep = st.all_tokens[-sp.repetition_context_size:] if sp.repetition_penalty != 1.0 else []
        outs = st.output_tokens if (sp.frequency_penalty or sp.presence_penalty) else []
        return rep, outs

    def _allow_mask(self, st):
        """numpy bool [V] of allowed tokens (grammar / tool constraint AND the
        reasoning budget), or None when every token is allowed."""
        c = st.req.token_constraint
        m = c.allowed_mask(self.V) if c is not None else None
        budget = st.extra.get("budget") if hasattr(st, "extra") else None
        if budget is not None:
            bm = budget.allowed_mask(self.V)
            if bm is not None:
                m = bm if m is None else (m & bm)
        return m

    @staticmethod
    def _forced(states):
        """(row, token) pairs whose next token is fixed (an exhausted reasoning
        budget forces the thought closer, even over a -inf logit)."""
        out = []
        for i, st in enumerate(states):
            b = st.extra.get("budget") if hasattr(st, "extra") else None
            f = b.forced() if b is not None else None
            if f is not None:
                out.append((i, f))
        return out

    # ------------------------------------------------------------------ main
    def sample(self, logits: torch.Tensor, states: list, out: torch.Tensor | None = None):
        """logits [R, V] fp32 for the rows in `states`. Returns (tokens int32
        tensor on logits' device, logprobs list or None)."""
        R = logits.shape[0]
        if R == 0:
            return torch.empty(0, dtype=torch.int32, device=logits.device), None
        want_lp = any(st.req.sampling.logprobs or st.req.sampling.top_logprobs for st in states)
        lp_info = None
        raw = logits.clone() if want_lp else None
        masks = [self._allow_mask(st) for st in states]
        need_proc = any(st.req.sampling.needs_processing for st in states) or any(m is not None for m in masks)
        all_greedy = all(st.req.sampling.greedy for st in states)
        # non-finite flags describe the model's logits, before bias / penalties / masks
        # add their -inf entries; the all-greedy unprocessed path gets them from the argmax pass
        fused_flags = logits.is_cuda and all_greedy and not need_proc
        self.last_flags = None if fused_flags else (~torch.isfinite(logits)).any(-1).to(torch.int32)
        if not logits.is_cuda:
            toks = self._sample_cpu(logits, states, masks)
        else:
            if need_proc:
                self._process_cuda(logits, states, masks)
            if all_greedy:
                if fused_flags:
                    self.last_flags = torch.empty(R, dtype=torch.int32, device=logits.device)
                toks = ops.argmax(logits, out=out, flags=self.last_flags if fused_flags else None)
            else:
                toks = self._sample_cuda(logits, states, out)
        forced = self._forced(states)
        if forced:
            idx = torch.tensor([i for i, _ in forced], dtype=torch.long, device=toks.device)
            toks[idx] = torch.tensor([t for _, t in forced], dtype=toks.dtype, device=toks.device)
        if want_lp:
            n_top = max(st.req.sampling.top_logprobs for st in states)
            tok_lp, top_ids, top_lp = ops.logprobs(raw, toks, n_top)
            lp_info = (tok_lp, top_ids, top_lp)
        return toks, lp_info

    def _process_cuda(self, logits, states, masks):
        R = len(states)
        dev = logits.device
        nb = [len(st.req.sampling.logit_bias) for st in states]
        reps, outs = zip(*[self._penalty_lists(st) for st in states])
        mb = max(1, max(nb))
        mr = max(1, max(len(r) for r in reps))
        mo = max(1, max(len(o) for o in outs))
        bias_ids = np.full((R, mb), -1, np.int32)
        bias_vals = np.zeros((R, mb), np.float32)
        rep_ids = np.full((R, mr), -1, np.int32)
        out_ids = np.full((R, mo), -1, np.int32)
        for i, st in enumerate(states):
            for j, (k, v) in enumerate(st.req.sampling.logit_bias.items()):
                bias_ids[i, j], bias_vals[i, j] = int(k), float(v)
            rep_ids[i, :len(reps[i])] = reps[i]
            out_ids[i, :len(outs[i])] = outs[i]
        sp = [st.req.sampling for st in states]
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt, non_blocking=False)
        mask_t = mrows = None
        if any(m is not None for m in masks):
            words = (self.V + 31) // 32
            mk = np.full((R, words), 0xFFFFFFFF, np.uint32)
            rows = np.zeros(R, np.int32)
            for i, m in enumerate(masks):
                if m is not None:
                    bits = np.packbits(np.pad(m.astype(np.uint8), (0, words * 32 - self.V)), bitorder="little")
                    mk[i] = bits.view(np.uint32)
                    rows[i] = 1
            mask_t = t(mk.view(np.int32), torch.int32)
            mrows = t(rows, torch.int32)
        ops.process_logits(
            logits, t(bias_ids, torch.int32), t(bias_vals, torch.float32), t(np.array(nb, np.int32), torch.int32),
            t(rep_ids, torch.int32), t(np.array([len(r) for r in reps], np.int32), torch.int32),
            t(np.array([p.repetition_penalty for p in sp], np.float32), torch.float32),
            t(out_ids, torch.int32), t(np.array([len(o) for o in outs], np.int32), torch.int32),
            t(np.array([p.frequency_penalty for p in sp], np.float32), torch.float32),
            t(np.array([p.presence_penalty for p in sp], np.float32), torch.float32), mask_t, mrows)

    def _sample_cuda(self, logits, states, out):
        dev = logits.device
        sp = [st.req.sampling for st in states]
        f = lambda xs, dt: torch.tensor(xs, dtype=dt).to(dev, non_blocking=False)
        keys = np.array([row_key(st) for st in states], dtype=np.uint64).view(np.int64)
        return ops.sample(logits, f([p.temperature for p in sp], torch.float32), f([p.top_k for p in sp], torch.int32),
                          f([p.top_p for p in sp], torch.float32), f([p.min_p for p in sp], torch.float32),
                          torch.from_numpy(keys).to(dev), f([st.gen_step for st in states], torch.int64), out=out)

    def _sample_cpu(self, logits, states, masks):
        toks = []
        for i, st in enumerate(states):
            sp = st.req.sampling
            rep, outs = self._penalty_lists(st)
            allow = torch.from_numpy(masks[i]) if masks[i] is not None else None
            lg = ref.process_logits_ref(logits[i], sp.logit_bias, rep, sp.repetition_penalty, outs,
                                        sp.frequency_penalty, sp.presence_penalty, allow)
            toks.append(ref.sample_ref(lg, sp.temperature, sp.top_k, sp.top_p, sp.min_p, row_key(st), st.gen_step))
        return torch.tensor(toks, dtype=torch.int32)

    @staticmethod
    def logprob_entries(lp_info, toks_host, states):
        if lp_info is None:
            return [None] * len(states)
        tok_lp, top_ids, top_lp = lp_info
        tok_lp = tok_lp.float().cpu().numpy()
        ti = top_ids.cpu().numpy() if top_ids is not None else None
        tl = top_lp.float().cpu().numpy() if top_lp is not None else None
        out = []
        for i, st in enumerate(states):
            sp = st.req.sampling
            if not (sp.logprobs or sp.top_logprobs):
                out.append(None)
                continue
            top = []
            if ti is not None and sp.top_logprobs:
                top = [(int(ti[i, j]), float(tl[i, j])) for j in range(sp.top_logprobs)]
            out.append(TokenLogprob(int(toks_host[i]), float(tok_lp[i]), top))
        return out
