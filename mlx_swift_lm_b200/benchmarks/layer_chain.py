"""In-graph cost of the decode step's op kinds: a chain of L layers' worth of
one op kind (distinct weights per layer, so every launch streams its weights
from HBM) captured in one CUDA graph and replayed, timed with CUDA events.

Serialized per-kernel timings (a profiler's launch list) miss what the
decode graph gets from programmatic dependent launch (each GEMM prefetches its
weights before the previous kernel ends) and add what it does not pay (a cold
launch per kernel). This bench times the kinds as the graph runs them:

    python -m mlx_swift_lm_b200.benchmarks.layer_chain [--layers 36] [--m 64] [--kinds qkv,o,gate_up,down,norm,chain]

Shapes are Qwen3-8B's (hidden 4096, 32 q / 8 kv heads of 128, intermediate
12288). "chain" runs qkv, o, add_rmsnorm, gate_up, down, add_rmsnorm per layer
(the GEMM and norm part of a decode layer, attention left out).
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops

SHAPES = {"qkv": (6144, 4096, "none"), "o": (4096, 4096, "none"), "gate_up": (24576, 4096, "swiglu"),
          "down": (4096, 12288, "none")}


def _time_graph(fn, reps: int = 20) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3)
    return sorted(ts)[len(ts) // 2]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--m", type=int, default=64)
    ap.add_argument("--kinds", default="qkv,o,gate_up,down,norm,chain")
    ap.add_argument("--hbm-gbs", type=float, default=0.0, help="roofline copy rate (default: measured peaks file)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    hbm = a.hbm_gbs
    if not hbm:
        try:
            with open("MEASURED_PEAKS.json") as f:
                hbm = float(json.load(f)["hbm_gbs"])
        except (OSError, KeyError, ValueError):
            hbm = 6650.0
    L, M = a.layers, a.m
    g = torch.Generator(device=dev).manual_seed(0)

    def rn(*s):
        return torch.empty(s, device=dev, dtype=torch.bfloat16).normal_(0, 0.02, generator=g)

    kinds = a.kinds.split(",")
    need = {k for k in kinds if k in SHAPES} | (set(SHAPES) if "chain" in kinds else set())
    W = {k: [rn(SHAPES[k][0], SHAPES[k][1]) for _ in range(L)] for k in need}
    x = rn(M, 4096)
    resid = rn(M, 4096)
    ln = torch.ones(4096, device=dev, dtype=torch.bfloat16)
    ys = {k: torch.empty(M, SHAPES[k][0] // (2 if SHAPES[k][2] == "swiglu" else 1), device=dev,
                         dtype=torch.bfloat16) for k in need}
    for k in kinds:
        if k in SHAPES:
            N, K, epi = SHAPES[k]
            xin = x if K == 4096 else rn(M, K)

            def fn(k=k, xin=xin, epi=epi):
                for li in range(L):
                    ops.gemm(xin, W[k][li], epi=epi, out=ys[k])

            t = _time_graph(fn)
            byt = L * (N * K * 2 + M * K * 2 + ys[k].numel() * 2)
            print(f"{k:8s} L={L} M={M} N={N} K={K}: {t / L * 1e6:7.2f} us/launch, {byt / t / 1e9:7.0f} GB/s, "
                  f"{byt / t / 1e9 / hbm:6.1%} of {hbm:.0f}", flush=True)
        elif k == "norm":
            out = torch.empty_like(x)

            def fn():
                for _ in range(2 * L):
                    ops.add_rmsnorm(resid, x, ln, 1e-6, out=out)

            t = _time_graph(fn)
            print(f"norm     {2 * L} add_rmsnorm launches: {t / (2 * L) * 1e6:7.2f} us/launch", flush=True)
        elif k == "chain":
            h = torch.empty_like(x)

            def fn():
                for li in range(L):
                    ops.gemm(h, W["qkv"][li], out=ys["qkv"])
                    ops.gemm(x, W["o"][li], out=ys["o"])
                    ops.add_rmsnorm(resid, ys["o"], ln, 1e-6, out=h)
                    ops.gemm(h, W["gate_up"][li], epi="swiglu", out=ys["gate_up"])
                    ops.gemm(ys["gate_up"], W["down"][li], out=ys["down"])
                    ops.add_rmsnorm(resid, ys["down"], ln, 1e-6, out=h)

            t = _time_graph(fn)
            byt = L * sum(SHAPES[k][0] * SHAPES[k][1] * 2 for k in SHAPES)
            print(f"chain    L={L} M={M}: {t * 1e3:8.3f} ms, {t / L * 1e6:7.2f} us/layer, weights "
                  f"{byt / t / 1e9:7.0f} GB/s, {byt / t / 1e9 / hbm:6.1%} of {hbm:.0f}", flush=True)


if __name__ == "__main__":
    main()
