"""One MoE expert layer (router top-k -> sort -> grouped GEMMs -> combine) of
the Qwen3-30B-A3B shape at T tokens: device time and weight bandwidth.

    python -m mlx_swift_lm_b200.benchmarks.moe_layer [--tokens 64]
"""
from __future__ import annotations

import argparse

import torch

from ..ops import _lib, moe
from ..ops.qlinear import QuantizedWeight


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--ffn", type=int, default=768)
    ap.add_argument("--bits", type=int, default=0, help="0 = bf16 experts; 4 / 8 = affine quantised, group 64")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    T, E, k, K, F = a.tokens, a.experts, a.topk, a.hidden, a.ffn
    torch.manual_seed(0)
    h = torch.randn(T, K, device=dev, dtype=torch.bfloat16)
    gu = torch.randn(E, 2 * F, K, device=dev, dtype=torch.bfloat16) * 0.02
    d = torch.randn(E, K, F, device=dev, dtype=torch.bfloat16) * 0.02
    if a.bits:
        gu = QuantizedWeight.stack_experts([QuantizedWeight.quantize(gu[e].float().cpu(), a.bits, 64)
                                            for e in range(E)]).to(dev)
        d = QuantizedWeight.stack_experts([QuantizedWeight.quantize(d[e].float().cpu(), a.bits, 64)
                                           for e in range(E)]).to(dev)
    w, idx = moe.route_topk(torch.randn(T, E, device=dev), k)
    for _ in range(3):
        moe.moe_experts(h, gu, d, w, idx)
    torch.cuda.synchronize()
    n = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        moe.moe_experts(h, gu, d, w, idx)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    used = torch.unique(idx).numel()
    per_expert = (gu.nbytes() + d.nbytes()) / E if a.bits else (2 * F * K + K * F) * 2
    byts = used * per_expert
    print(f"moe bits={a.bits or 16} T={T} E={E} k={k} {ms * 1e3:.1f} us/layer experts used {used} weight bytes {byts / 1e9:.2f} GB "
          f"{byts / ms / 1e6:.0f} GB/s status {_lib.read_status()}", flush=True)


if __name__ == "__main__":
    main()
