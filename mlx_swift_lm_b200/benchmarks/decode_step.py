"""Eager decode step of a named model shape at B rows with a synthetic paged
KV state of `ctx` tokens per row (no prefill needed): prints the step time.
With --profile the last step runs between cudaProfilerStart/Stop, so
``ncu --profile-from-start off`` captures exactly one step's kernels.

    python -m mlx_swift_lm_b200.benchmarks.decode_step --model qwen3_8b --batch 64 --ctx 1100 [--layers 2] [--profile]
"""
from __future__ import annotations

import argparse

import torch

from .. import DecoderLM, ops
from ..kv.paged import PagedKVCache, SequenceKV
from ..models import config as mcfg
from ..models.batch import ForwardBatch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3_8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1100)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (smaller profiles)")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--profile", action="store_true")
    a = ap.parse_args(argv)
    cfg = getattr(mcfg, a.model)()
    if a.layers:
        cfg.num_layers = a.layers
    dev = torch.device("cuda", 0)
    m = DecoderLM(cfg, dev, torch.bfloat16).init_random(0)
    B, ctx = a.batch, a.ctx
    kv = PagedKVCache.for_model(m, max_tokens=B * (ctx + 32))
    seqs = []
    for _ in range(B):
        s = SequenceKV(kv)
        s.ensure(ctx + 1)
        s.num_tokens = ctx
        seqs.append(s)
    maxp = max(len(s.pages) for s in seqs)
    pt = torch.zeros(B, maxp, dtype=torch.int32)
    for b, s in enumerate(seqs):
        pt[b, :len(s.pages)] = torch.tensor(s.pages)
    fb = ForwardBatch(input_ids=torch.randint(0, cfg.vocab_size, (B,), dtype=torch.int32, device=dev),
                      positions=torch.full((B,), ctx, dtype=torch.int32, device=dev),
                      slots=torch.tensor([s.slot(ctx) for s in seqs], dtype=torch.int64, device=dev), num_decode=B,
                      dec_page_table=pt.to(dev), dec_seq_lens=torch.full((B,), ctx + 1, dtype=torch.int32, device=dev),
                      dec_max_parts=(ctx + 256) // 256)
    out = torch.empty(B, dtype=torch.int32, device=dev)

    def step():
        lg = m.forward(fb, kv)
        ops.argmax(lg, out=out)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    print(f"eager step {e0.elapsed_time(e1) / a.steps:.3f} ms (model={a.model}, B={B}, ctx={ctx}, "
          f"layers={cfg.num_layers})", flush=True)
    if a.profile:
        torch.cuda.profiler.start()
        step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()
