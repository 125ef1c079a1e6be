"""One GEMM shape, bf16 or affine-quantised weights, for kernel profiling:
3 warm-up launches then `--reps` launches between cudaProfilerStart/Stop.

    python -m mlx_swift_lm_b200.benchmarks.gemm_one --m 16 --n 6144 --k 4096 --bits 4 [--reps 3]
"""
from __future__ import annotations

import argparse

import torch

from .. import ops
from ..ops.qlinear import QuantizedWeight


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=16)
    ap.add_argument("--n", type=int, default=6144)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--bits", type=int, default=0)
    ap.add_argument("--gs", type=int, default=64)
    ap.add_argument("--epi", default="none")
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    w = torch.randn(a.n, a.k) * 0.02
    W = w.to(dev, torch.bfloat16) if a.bits == 0 else QuantizedWeight.quantize(w, a.bits, a.gs).to(dev)
    x = torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        ops.gemm(x, W, epi=a.epi)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    e0.record()
    for _ in range(a.reps):
        ops.gemm(x, W, epi=a.epi)
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"gemm M={a.m} N={a.n} K={a.k} bits={a.bits} {e0.elapsed_time(e1) / a.reps * 1e3:.1f} us/launch "
          f"(back to back)", flush=True)


if __name__ == "__main__":
    main()
