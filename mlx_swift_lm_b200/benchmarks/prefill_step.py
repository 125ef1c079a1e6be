"""Eager prefill step of a named model shape: `batch` fresh prompts of `len`
tokens each as one flattened chunked-prefill batch (paged KV), timed with
CUDA events; --profile runs one more step between cudaProfilerStart/Stop.

    python -m mlx_swift_lm_b200.benchmarks.prefill_step --model qwen3_8b --batch 4 --len 2048 [--layers 2] [--profile]
"""
from __future__ import annotations

import argparse

import numpy as np
import torch

from .. import DecoderLM
from ..kv.paged import PagedKVCache, SequenceKV
from ..models import config as mcfg
from ..models.batch import ForwardBatch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3_8b")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--len", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--profile", action="store_true")
    a = ap.parse_args(argv)
    cfg = getattr(mcfg, a.model)()
    if a.layers:
        cfg.num_layers = a.layers
    dev = torch.device("cuda", 0)
    m = DecoderLM(cfg, dev, torch.bfloat16).init_random(0)
    B, L = a.batch, a.len
    kv = PagedKVCache.for_model(m, max_tokens=B * (L + 16))
    seqs = []
    for _ in range(B):
        s = SequenceKV(kv)
        s.ensure(L)
        seqs.append(s)
    maxp = max(len(s.pages) for s in seqs)
    pt = np.zeros((B, maxp), np.int32)
    for i, s in enumerate(seqs):
        pt[i, :len(s.pages)] = s.pages
    cu = [i * L for i in range(B + 1)]
    ids = torch.randint(0, cfg.vocab_size, (B * L,), dtype=torch.int32)
    fb = ForwardBatch(input_ids=ids.to(dev), positions=torch.arange(L, dtype=torch.int32).repeat(B).to(dev),
                      slots=torch.tensor(sum((s.slots(0, L) for s in seqs), []), dtype=torch.int64, device=dev),
                      num_decode=0)
    fb.pf_cu_q = torch.tensor(cu, dtype=torch.int32, device=dev)
    fb.pf_cu_q_host = cu
    fb.pf_pos0 = torch.zeros(B, dtype=torch.int32, device=dev)
    fb.pf_page_table = torch.from_numpy(pt).to(dev)
    fb.logit_idx = torch.tensor([c - 1 for c in cu[1:]], dtype=torch.int64, device=dev)
    for _ in range(2):
        m.forward(fb, kv)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        m.forward(fb, kv)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    print(f"prefill step {ms:.2f} ms for {B}x{L} tokens ({B * L / ms * 1e3:.0f} tok/s, model={a.model}, "
          f"layers={cfg.num_layers})", flush=True)
    if a.profile:
        torch.cuda.profiler.start()
        m.forward(fb, kv)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()
