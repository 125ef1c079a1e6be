"""Pipeline parallelism: contiguous layer ranges per stage, hidden states sent
stage to stage with point-to-point sends (NCCL on GPUs, gloo on CPU), the
batch cut into microbatches so stages work concurrently.

Each rank of a pipeline group owns layers [lo, hi) of the model (stage 0 also
the embedding, the last stage the final norm and LM head) and a paged KV
cache for its own layers only. Every rank runs the same scheduler on the same
requests, so all stages build identical forward batches; the last stage
samples and broadcasts the tokens (EngineV2 does this when
``model.pp_stages > 1``).

Overlap: a step's rows are split into microbatches; a stage runs microbatch
j, posts an asynchronous send of its output, and continues with microbatch
j+1 while the next stage computes j. Tensor parallelism composes: each stage
can itself be a TP group (the model's `tp`).
"""
from __future__ import annotations

import copy

import torch
import torch.distributed as dist

from ..models.batch import ForwardBatch
from ..models.decoder import DecoderLM, TensorParallel


def stage_layers(num_layers: int, stages: int) -> list[tuple[int, int]]:
    """Balanced contiguous layer ranges (earlier stages take the remainder)."""
    base, extra = divmod(num_layers, stages)
    out, lo = [], 0
    for s in range(stages):
        n = base + (1 if s < extra else 0)
        out.append((lo, lo + n))
        lo += n
    return out


class PipelineParallel:
    """Pipeline context of a rank: its stage, the ranks of its neighbours and
    of the last stage (global ranks), and the group the tokens are broadcast
    in."""

    def __init__(self, stage: int, stages: int, ranks: list[int], group=None):
        self.stage, self.stages, self.ranks, self.group = stage, stages, list(ranks), group
        self.prev = ranks[stage - 1] if stage > 0 else None
        self.next = ranks[stage + 1] if stage + 1 < stages else None
        self.last = ranks[-1]

    @property
    def is_first(self) -> bool:
        return self.stage == 0

    @property
    def is_last(self) -> bool:
        return self.stage == self.stages - 1


class PipelinedDecoderLM(DecoderLM):
    """The layers [lo, hi) of a decoder (one pipeline stage). `forward`
    returns logits on the last stage and None elsewhere."""

    def __init__(self, cfg, pp: PipelineParallel, device="cpu", dtype=torch.float32, tp: TensorParallel | None = None,
                 microbatches: int = 0):
        self.full_cfg = cfg
        self.pp = pp
        self.layer_range = stage_layers(cfg.num_layers, pp.stages)[pp.stage]
        super().__init__(cfg, device, dtype, tp)
        self.microbatches = microbatches or pp.stages

    @property
    def pp_stages(self) -> int:
        return self.pp.stages

    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True, keep_layers=None):
        super().init_random(seed, std, with_embeddings, keep_layers=self.layer_range)
        self._to_stage_cfg()
        if not self.pp.is_first and not self.pp.is_last:
            self.embed = self.lm_head = None
        elif not self.pp.is_first and self.lm_head is self.embed:
            pass  # tied head: the last stage keeps the table for its logits
        return self

    def adopt_layers(self, full: DecoderLM):
        """Take this stage's share of an already built full model."""
        lo, hi = self.layer_range
        self.layers = full.layers[lo:hi]
        self.embed, self.norm, self.lm_head = full.embed, full.norm, full.lm_head
        self._to_stage_cfg()
        return self

    def _to_stage_cfg(self):
        lo, hi = self.layer_range
        c = copy.deepcopy(self.full_cfg)
        c.num_layers = hi - lo
        if c.layer_windows:
            c.layer_windows = list(self.full_cfg.layer_windows)[lo:hi]
        c.moe_layers = [self.full_cfg.is_moe(i) for i in range(lo, hi)]
        self.cfg = c

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        pp = self.pp
        mbs = split_rows(fb, self.microbatches)
        pending, outs = [], []
        H = self.full_cfg.hidden_size
        for mb in mbs:
            if pp.is_first:
                x_in = None
            else:
                x_in = torch.empty(mb.num_tokens, H, dtype=self.dtype, device=self.device)
                dist.recv(x_in, src=pp.prev)
            if pp.is_last:
                outs.append(super().forward(mb, kv, return_hidden=return_hidden, inputs_embeds=x_in,
                                            return_both=return_both))
            else:
                y = super().forward(mb, kv, inputs_embeds=x_in, return_residual=True).contiguous()
                pending.append((dist.isend(y, dst=pp.next), y))
        for req, _ in pending:
            req.wait()
        if not pp.is_last:
            return None
        if return_both:
            return torch.cat([o[0] for o in outs], 0), torch.cat([o[1] for o in outs], 0)
        return torch.cat(outs, 0)

    def forward_decode_tokens(self, fb, kv, out, out2=None, flags=None):
        from .. import ops

        logits = self.forward(fb, kv)
        if self.pp.is_last:
            ops.argmax(logits, out=out, out2=out2)
        dist.broadcast(out, src=self.pp.last, group=self.pp.group)
        if out2 is not None:
            out2.copy_(out)
        return out


def split_rows(fb: ForwardBatch, n: int) -> list[ForwardBatch]:
    """Cut a forward batch into at most n microbatches of whole rows (decode
    rows first, as the layout requires); logit rows follow their tokens."""
    nd = fb.num_decode
    pf_cu = fb.pf_cu_q_host or [0]
    rows = [(1, True)] * nd + [(pf_cu[i + 1] - pf_cu[i], False) for i in range(len(pf_cu) - 1)]
    R = len(rows)
    if n <= 1 or R <= 1:
        return [fb]
    n = min(n, R)
    total = fb.num_tokens
    # balance by tokens: cut where the running count passes k * total / n
    cuts, run, k = [0], 0, 1
    for i, (t, _) in enumerate(rows):
        run += t
        if k < n and run >= k * total / n and i + 1 < R:
            cuts.append(i + 1)
            k += 1
    cuts.append(R)
    logit_host = fb.logit_idx_host if fb.logit_idx is not None else None
    if fb.logit_idx is not None and logit_host is None:
        logit_host = fb.logit_idx.tolist()
    out = []
    tok_start = [0]
    for t, _ in rows:
        tok_start.append(tok_start[-1] + t)
    for a, b in zip(cuts[:-1], cuts[1:]):
        t0, t1 = tok_start[a], tok_start[b]
        d0, d1 = min(a, nd), min(b, nd)  # decode rows in [a, b)
        p0, p1 = max(a, nd) - nd, max(b, nd) - nd  # prefill rows
        mb = ForwardBatch(input_ids=fb.input_ids[t0:t1], positions=fb.positions[t0:t1], slots=fb.slots[t0:t1],
                          num_decode=d1 - d0)
        if d1 > d0:
            mb.dec_page_table = fb.dec_page_table[d0:d1]
            mb.dec_seq_lens = fb.dec_seq_lens[d0:d1]
            mb.dec_max_parts = fb.dec_max_parts
        if p1 > p0:
            base = pf_cu[p0]
            cu = [c - base for c in pf_cu[p0:p1 + 1]]
            mb.pf_cu_q_host = cu
            mb.pf_cu_q = torch.tensor(cu, dtype=torch.int32, device=fb.input_ids.device)
            mb.pf_pos0 = fb.pf_pos0[p0:p1]
            mb.pf_page_table = fb.pf_page_table[p0:p1]
        if logit_host is not None:
            sel = [i - t0 for i in logit_host if t0 <= i < t1]
            mb.logit_idx = torch.tensor(sel, dtype=torch.int64, device=fb.input_ids.device)
            mb.logit_idx_host = sel
        out.append(mb)
    return out
