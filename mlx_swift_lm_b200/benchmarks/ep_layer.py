"""One expert-parallel MoE layer of the Qwen3-30B-A3B shape across the ranks
of a torchrun job: fused dispatch/combine over symmetric memory vs the NCCL
all-to-all baseline, device time (CUDA events, max over ranks).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m mlx_swift_lm_b200.benchmarks.ep_layer [--tokens 64]

Bytes over NVLink per rank and direction: T * k * (W-1)/W rows of H bf16 for
the dispatch and again for the return.
"""
from __future__ import annotations

import argparse
import os

import torch
import torch.distributed as dist

from ..ops import reference as ref
from ..ops.qlinear import QuantizedWeight
from ..parallel.expert import ExpertParallel


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=64, help="tokens per rank")
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--ffn", type=int, default=768)
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--reps", type=int, default=50)
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    E, k, H, F, T = a.experts, a.topk, a.hidden, a.ffn, a.tokens
    El = E // world
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    gu = [ref.interleave_gate_up(torch.randn(F, H, device=dev) * 0.02, torch.randn(F, H, device=dev) * 0.02)
          for _ in range(El)]
    d = [torch.randn(H, F, device=dev) * 0.02 for _ in range(El)]
    if a.bits:
        gu = QuantizedWeight.stack_experts([QuantizedWeight.quantize_device(t, a.bits, 64) for t in gu])
        d = QuantizedWeight.stack_experts([QuantizedWeight.quantize_device(t, a.bits, 64) for t in d])
    else:
        gu, d = torch.stack(gu).to(torch.bfloat16), torch.stack(d).to(torch.bfloat16)
    h = torch.randn(T, H, device=dev, dtype=torch.bfloat16, generator=g)
    lg = torch.randn(T, E, device=dev, generator=g)
    res = {}
    for impl in ("fused", "a2a"):
        ep = ExpertParallel(E, k, H, rank, world, dist.group.WORLD, dev, max_tokens=T, impl=impl)

        def step():
            ep.begin_step()
            return ep.moe(h, lg, gu, d, tokens_max=T)

        for _ in range(5):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.reps):
            step()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / a.reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[impl] = t.item() * 1e3
        dist.barrier()
        ep.close()
    if rank == 0:
        byts = 2 * T * k * (world - 1) / world * H * 2
        print(f"ep layer W={world} T={T}/rank k={k} bits={a.bits or 16}: fused {res['fused']:.1f} us, "
              f"nccl all-to-all {res['a2a']:.1f} us; NVLink bytes/rank/dir {byts / 1e6:.2f} MB "
              f"-> {byts / (res['fused'] * 1e-6) / 1e9:.0f} GB/s at the fused time")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
