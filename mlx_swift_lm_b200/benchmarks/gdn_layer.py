"""One Gated DeltaNet layer body (conv + gates, delta-rule recurrence, gated
norm; the projections excluded) of the Qwen3-Next shape: decode steps of B
rows and one prefill chunk, device time and the recurrent-state bandwidth.

    python -m mlx_swift_lm_b200.benchmarks.gdn_layer [--rows 64] [--chunk 2048]
    python -m mlx_swift_lm_b200.benchmarks.gdn_layer --mamba   # Mamba-2, NemotronH-8B mixer shape

Decode reads and writes every row's fp32 state once per step, so its
roofline is 2 * B * Hv * Dv * Dk * 4 bytes at HBM bandwidth.
"""
from __future__ import annotations

import argparse

import torch

from ..ops.gdn import GdnRows, gdn_layer


def _time(fn, reps):
    for _ in range(3):
        fn()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    tot = 0.0
    for _ in range(reps):
        flush.zero_()  # evict the state from L2 between steps
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / reps


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--chunk", type=int, default=2048)
    ap.add_argument("--hk", type=int, default=16)
    ap.add_argument("--hv", type=int, default=32)
    ap.add_argument("--dk", type=int, default=128)
    ap.add_argument("--dv", type=int, default=128)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--mamba", action="store_true",
                    help="Mamba-2 mixer body (n_groups 8, state 128, 128 heads of 64)")
    a = ap.parse_args(argv)
    if a.mamba:
        return _mamba(a)
    dev = torch.device("cuda", 0)
    Hk, Dk, Hv, Dv, B = a.hk, a.dk, a.hv, a.dv, a.rows
    C = 2 * Hk * Dk + Hv * Dv
    torch.manual_seed(0)
    conv_w = torch.randn(C, 4, device=dev) * 0.3
    A_log, dt_bias = torch.rand(Hv, device=dev) * 2, torch.randn(Hv, device=dev)
    norm_w = torch.ones(Dv, device=dev, dtype=torch.bfloat16)
    cs = torch.zeros(B + 1, 3, C, device=dev, dtype=torch.bfloat16)
    ss = torch.zeros(B + 1, Hv, Dv, Dk, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    P = torch.randn(B, C + Hv * Dv + 2 * Hv, device=dev, dtype=torch.bfloat16)
    rows = GdnRows(torch.arange(B + 1, **i32), torch.zeros(B, **i32), torch.arange(B, **i32))
    ms = _time(lambda: gdn_layer(P, rows, cs, ss, conv_w, A_log, dt_bias, norm_w, Hk, Dk, Hv, Dv, 1e-6), a.reps)
    sbytes = 2 * B * Hv * Dv * Dk * 4
    print(f"gdn decode B={B} Hk={Hk} Hv={Hv} D={Dk}: {ms * 1e3:.1f} us/layer, state traffic {sbytes / 1e6:.1f} MB "
          f"-> {sbytes / (ms * 1e-3) / 1e12:.2f} TB/s")
    T = a.chunk
    Pc = torch.randn(T, C + Hv * Dv + 2 * Hv, device=dev, dtype=torch.bfloat16)
    rows1 = GdnRows(torch.tensor([0, T], **i32), torch.ones(1, **i32), torch.zeros(1, **i32), [0, T])
    ms = _time(lambda: gdn_layer(Pc, rows1, cs, ss, conv_w, A_log, dt_bias, norm_w, Hk, Dk, Hv, Dv, 1e-6), 5)
    print(f"gdn prefill one row T={T}: {ms:.3f} ms/layer ({T / ms * 1e3:.0f} tok/s)")


def _mamba(a):
    from ..ops.gdn import mamba_layer

    dev = torch.device("cuda", 0)
    G, N, H, Pd, B = 8, 128, 128, 64, a.rows
    C = 2 * G * N + H * Pd
    torch.manual_seed(0)
    conv_w, conv_b = torch.randn(C, 4, device=dev) * 0.3, torch.zeros(C, device=dev)
    A_log, dt_bias, D = torch.rand(H, device=dev) * 2, torch.randn(H, device=dev), torch.ones(H, device=dev)
    norm_w = torch.ones(H * Pd, device=dev, dtype=torch.bfloat16)
    cs = torch.zeros(B + 1, 3, C, device=dev, dtype=torch.bfloat16)
    ss = torch.zeros(B + 1, H, Pd, N, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    P = torch.randn(B, C + H * Pd + H, device=dev, dtype=torch.bfloat16)
    rows = GdnRows(torch.arange(B + 1, **i32), torch.zeros(B, **i32), torch.arange(B, **i32))
    lim = (0.0, float("inf"))
    ms = _time(lambda: mamba_layer(P, rows, cs, ss, conv_w, conv_b, A_log, dt_bias, D, norm_w, G, N, H, Pd, 1e-5,
                                   H * Pd // G, lim), a.reps)
    sbytes = 2 * B * H * Pd * N * 4
    print(f"mamba2 decode B={B} G={G} N={N} H={H} P={Pd}: {ms * 1e3:.1f} us/layer, state traffic "
          f"{sbytes / 1e6:.1f} MB -> {sbytes / (ms * 1e-3) / 1e12:.2f} TB/s")
    T = a.chunk
    Pc = torch.randn(T, C + H * Pd + H, device=dev, dtype=torch.bfloat16)
    rows1 = GdnRows(torch.tensor([0, T], **i32), torch.ones(1, **i32), torch.zeros(1, **i32), [0, T])
    ms = _time(lambda: mamba_layer(Pc, rows1, cs, ss, conv_w, conv_b, A_log, dt_bias, D, norm_w, G, N, H, Pd, 1e-5,
                                   H * Pd // G, lim), 5)
    print(f"mamba2 prefill one row T={T}: {ms:.3f} ms/layer ({T / ms * 1e3:.0f} tok/s)")


if __name__ == "__main__":
    main()
