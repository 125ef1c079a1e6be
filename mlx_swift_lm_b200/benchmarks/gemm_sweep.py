"""GEMM sweep over the decode/prefill shapes of a model: bf16 weights and
affine-quantised (4/8-bit) weights through the tcgen05 kernels. Each point is
the median of 10 CUDA-event timings with a 256 MiB L2 flush before each.

    python -m mlx_swift_lm_b200.benchmarks.gemm_sweep [--ms 1,16,64,128,2048] [--bits 0,4,8] [--role prefill]
                                                      [--splits 1,2,4,8]

--role prefill times the launch prefill rows get in a serving step (no split-K;
256 x 256 tiles above 128 rows); the default times the (N, K)-chosen split-K
launch that decode rows get; --splits times forced split-K counts instead.
"""
from __future__ import annotations

import argparse

import torch

from .. import ops
from ..ops.qlinear import QuantizedWeight

QWEN3_8B = [(6144, 4096, "none"), (4096, 4096, "none"), (24576, 4096, "swiglu"), (4096, 12288, "none"),
            (151936, 4096, "f32")]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ms", default="1,16,64,128,512,2048")
    ap.add_argument("--bits", default="0", help="0 = bf16 weights; 4 / 8 = affine quantised, group 64")
    ap.add_argument("--role", default="decode", choices=["decode", "prefill"])
    ap.add_argument("--splits", default="", help="forced split-K counts (bf16 weights), e.g. 1,2,3,4,6,8")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    sps = [int(v) for v in a.splits.split(",")] if a.splits else [1 if a.role == "prefill" else 0]
    for bits in [int(b) for b in a.bits.split(",")]:
        for N, K, epi in QWEN3_8B:
            w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
            W = w if bits == 0 else QuantizedWeight.quantize(w.float().cpu(), bits, 64).to(dev)
            wbytes = N * K * 2 if bits == 0 else W.nbytes()
            for M, sp in [(int(x), sp) for x in a.ms.split(",") for sp in sps]:
                x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
                for _ in range(3):
                    ops.gemm(x, W, epi=epi, splits=sp)
                ts = []
                for _ in range(10):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    ops.gemm(x, W, epi=epi, splits=sp)
                    e1.record()
                    torch.cuda.synchronize()
                    ts.append(e0.elapsed_time(e1))
                t = sorted(ts)[len(ts) // 2] * 1e-3
                out_b = M * N * (4 if epi == "f32" else 2) // (2 if epi == "swiglu" else 1)
                byt = wbytes + M * K * 2 + out_b
                tag = f"S={sp}" if a.splits else a.role
                print(f"{tag} w={'bf16' if bits == 0 else f'q{bits}':4s} M={M:5d} N={N:6d} K={K:5d} {epi:6s} "
                      f"{t * 1e6:9.1f} us {byt / t / 1e9:7.0f} GB/s {2 * M * N * K / t / 1e12:7.1f} TFLOP/s",
                      flush=True)


if __name__ == "__main__":
    main()
