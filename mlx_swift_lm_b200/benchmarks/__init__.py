"""Benchmark drivers (decode-step kernel breakdown, GEMM sweeps, MoE layer).

Parity: the reference's bench drivers (BenchCBv2 and friends) measure engine
throughput and per-kernel costs on real weights; these drive the same hot
paths on random weights of a named architecture, timed with CUDA events.
Each is runnable as ``python -m mlx_swift_lm_b200.benchmarks.<name>``.
"""
