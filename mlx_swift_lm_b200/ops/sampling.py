"""Sampling ops: logits processing, sampling, argmax, logprobs."""
from __future__ import annotations

import torch

from . import _lib
from . import reference as ref


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None, out2: torch.Tensor | None = None,
           flags: torch.Tensor | None = None):
    """Greedy tokens [B] int32 from fp32 logits [B, V]. `out2` optionally
    receives a second copy (e.g. the next decode step's input ids); `flags`
    (int32 [B]) receives 1 for rows holding a NaN or infinite logit, from the
    same pass over the logits."""
    if not logits.is_cuda:
        lf = logits.float()
        y = torch.nan_to_num(lf, nan=-float("inf")).argmax(-1).to(torch.int32)
        if out is not None:
            out.copy_(y)
            y = out
        if out2 is not None:
            out2.copy_(y)
        if flags is not None:
            flags.copy_((~torch.isfinite(lf)).any(-1).to(torch.int32))
        return y
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    rc = _lib.lib().b200_argmax(logits.data_ptr(), logits.stride(0), B, V, out.data_ptr(), _lib.ptr(out2),
                                _lib.ptr(flags), _lib.stream_ptr(logits.device))
    _lib.check(rc, "argmax")
    _lib.count(1)
    return out


CONF_CHUNK = 8192  # logits per CTA of the split greedy-confidence pass


def argmax_confidence(logits: torch.Tensor):
    """(greedy tokens [B] int32, softmax probability of that token [B] fp32,
    max logit [B] fp32) of fp32 logits [B, V] in one pass (mask-diffusion
    commit scores)."""
    if not logits.is_cuda:
        lf = logits.float()
        mx, tok = lf.max(-1)
        tok = lf.argmax(-1)
        conf = torch.exp(mx - torch.logsumexp(lf, -1))
        return tok.to(torch.int32), conf, mx
    B, V = logits.shape
    tok = torch.empty(B, dtype=torch.int32, device=logits.device)
    conf = torch.empty(B, dtype=torch.float32, device=logits.device)
    mx = torch.empty(B, dtype=torch.float32, device=logits.device)
    # Large vocabularies are split into chunks of about CONF_CHUNK logits, a CTA per
    # (row, chunk), and the triples are merged per row in chunk order. The split
    # depends on V only, never on B, so a row's confidence is bit-identical whatever
    # batch it is scored in (the diffusion engine thresholds it and picks maxima).
    nsplit = -(-V // CONF_CHUNK) if V > CONF_CHUNK else 1
    scratch = torch.empty(3 * B * nsplit, dtype=torch.float32, device=logits.device) if nsplit > 1 else None
    rc = _lib.lib().b200_argmax_conf(logits.data_ptr(), logits.stride(0), B, V, tok.data_ptr(), conf.data_ptr(),
                                     mx.data_ptr(), _lib.ptr(scratch), nsplit, _lib.stream_ptr(logits.device))
    _lib.check(rc, "argmax_conf")
    _lib.count(2 if nsplit > 1 else 1)
    return tok, conf, mx


def process_logits(logits, bias_ids=None, bias_vals=None, n_bias=None, rep_ids=None, n_rep=None, rep_penalty=None,
                   out_ids=None, n_out=None, freq=None, pres=None, allow_mask=None, mask_rows=None):
    """In-place logit bias, repetition / frequency / presence penalties and token mask (CUDA)."""
    B, V = logits.shape
    rc = _lib.lib().b200_logits_process(
        logits.data_ptr(), logits.stride(0), B, V, _lib.ptr(bias_ids), _lib.ptr(bias_vals), _lib.ptr(n_bias),
        bias_ids.stride(0) if bias_ids is not None else 0, _lib.ptr(rep_ids), _lib.ptr(n_rep),
        rep_ids.stride(0) if rep_ids is not None else 0, _lib.ptr(rep_penalty), _lib.ptr(out_ids), _lib.ptr(n_out),
        out_ids.stride(0) if out_ids is not None else 0, _lib.ptr(freq), _lib.ptr(pres), _lib.ptr(allow_mask),
        allow_mask.stride(0) if allow_mask is not None else 0, _lib.ptr(mask_rows), _lib.stream_ptr(logits.device))
    _lib.check(rc, "logits_process")
    _lib.count(1)
    return logits


def sample(logits, temperature, top_k, top_p, min_p, keys, steps, out=None, out2=None, out_logit=None, flags=None):
    """Per-row temperature / top-k / top-p / min-p + Gumbel-max draw (CUDA);
    `flags` (int32 [B]) receives the rows' non-finite-logit flags."""
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    rc = _lib.lib().b200_sample(logits.data_ptr(), logits.stride(0), B, V, temperature.data_ptr(), top_k.data_ptr(),
                                top_p.data_ptr(), min_p.data_ptr(), keys.data_ptr(), steps.data_ptr(), out.data_ptr(),
                                _lib.ptr(out2), _lib.ptr(out_logit), _lib.ptr(flags), _lib.stream_ptr(logits.device))
    _lib.check(rc, "sample")
    _lib.count(1)
    return out


def logprobs(logits, tokens, n_top: int = 0):
    """Raw log-softmax: logprob of tokens[b] and top-n (ids, logprobs)."""
    B, V = logits.shape
    if not logits.is_cuda:
        lp = torch.log_softmax(logits.float(), dim=-1)
        tok_lp = lp.gather(1, tokens.long()[:, None])[:, 0] if tokens is not None else None
        if n_top > 0:
            v, i = torch.topk(lp, n_top, dim=-1)
            return tok_lp, i.to(torch.int32), v
        return tok_lp, None, None
    out_lp = torch.empty(B, dtype=torch.float32, device=logits.device)
    top_ids = torch.empty((B, max(n_top, 1)), dtype=torch.int32, device=logits.device)
    top_lp = torch.empty((B, max(n_top, 1)), dtype=torch.float32, device=logits.device)
    rc = _lib.lib().b200_logprobs(logits.data_ptr(), logits.stride(0), B, V, _lib.ptr(tokens), n_top,
                                  out_lp.data_ptr(), top_ids.data_ptr(), top_lp.data_ptr(),
                                  _lib.stream_ptr(logits.device))
    _lib.check(rc, "logprobs")
    _lib.count(1)
    return (out_lp if tokens is not None else None), (top_ids if n_top else None), (top_lp if n_top else None)


def sample_rows_cpu(logits, params_rows):
    """CPU oracle for a batch: params_rows is a list of dicts with keys
    temperature, top_k, top_p, min_p, key, step (after processing)."""
    out = []
    for b, p in enumerate(params_rows):
        out.append(ref.sample_ref(logits[b], p["temperature"], p.get("top_k", 0), p.get("top_p", 1.0),
                                  p.get("min_p", 0.0), p.get("key", 0), p.get("step", 0)))
    return torch.tensor(out, dtype=torch.int32)
