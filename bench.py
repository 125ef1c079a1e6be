#!/usr/bin/env python3
"""Headline benchmark: decode tok/s at 64 concurrent streams (+ p50 TTFT / ITL).

Config: Qwen3-8B-shape dense decoder, bf16, random-init
N(0, 0.02) weights, paged KV (page 16), 64 requests with prompt lengths
uniform in [128, 2048] (random token ids), 256 output tokens each, greedy.
Tensor parallel over all GPUs of the run (tp = N).

Measurement:
  * prefill phase: all 64 requests are submitted and the engine steps until
    every row decodes; TTFT p50 comes from the engine's per-request timing.
  * ``value`` (kernel-only): K replays of the captured 64-row decode-step CUDA
    graph (full forward + sampling at the real context lengths), after W
    warm-up replays, bracketed by barrier + synchronize, timed with CUDA
    events; max over ranks. Inputs (weights 16 GB + KV) exceed L2.
  * ``e2e``: K more decode steps through the public engine API
    (``EngineV2.step``), whose every step copies its inputs host->device from
    pinned memory and reads the sampled tokens back; wall clock with
    synchronize on both sides; max over ranks. ITL p50 from these steps.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (box, device-timed, max over ranks) @64 streams; p50 TTFT, ITL"
BASELINE_VALUE = None  # BASELINE.md publishes no 64-stream number on any hardware


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3_8b")
    ap.add_argument("--streams", type=int, default=64)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=2048)
    ap.add_argument("--out-tokens", type=int, default=256)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (debug only; invalid for the headline)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tp-mode", default="nccl", choices=["fused", "nccl"],
                    help="tensor-parallel collectives: fused symmetric-memory kernels or NCCL all-reduce")
    ap.add_argument("--quant-experts", type=int, default=0, help="MLX affine bits for MoE experts (0 = bf16)")
    ap.add_argument("--quant-dense", type=int, default=0, help="MLX affine bits for dense projections (0 = bf16)")
    ap.add_argument("--mtp", type=int, default=0, help="MTP draft depth k (0 = off); acceptance: seeded Bernoulli(0.7)")
    ap.add_argument("--pp", type=int, default=1, help="pipeline stages (world = pp x tp); stages exchange hidden "
                                                     "states with NCCL p2p")
    ap.add_argument("--kv-fp8", action="store_true", help="fp8-e4m3 paged KV with per-head scales")
    ap.add_argument("--ep", type=int, default=1, help="expert-parallel ranks (world = ep): MoE experts split whole "
                                                      "across ranks, attention data-parallel over the rows")
    ap.add_argument("--ep-mode", default="fused", choices=["fused", "a2a"],
                    help="fused: dispatch/combine kernels over symmetric memory; a2a: NCCL all_to_all baseline")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi SM clock / throttle-reason sampler for the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


EP_MAX_TOKENS = 8192  # tokens per step (all ranks) with expert parallelism; sizes the EP receive buffers


def _par(args, world):
    if args.pp > 1:
        return f"pp{args.pp}xtp{world // args.pp}"
    if args.ep > 1:
        return f"ep{args.ep} ({args.ep_mode} dispatch/combine, data-parallel attention)"
    return f"tp{world}" + (f" ({args.tp_mode} collectives)" if world > 1 else "")


def reference_arm(args):
    print(json.dumps({"impl": "reference", "metric": METRIC,
                      "unavailable": "the reference (Layr-Labs/mlx-swift-lm) is a Swift/MLX/Metal package for Apple "
                                     "GPUs: it has no setup.py/pyproject (pip install fails) and no CUDA path"}))
    return 0


def _mtp_measure(args, eng, mtp, streams, dev, world, rank, ttfts, prefill_s, cfg, barrier, ClockSampler, local, _lib):
    """MTP rounds are eager (draft steps + one batched verify): value = tokens
    emitted per second over K engine steps timed with CUDA events on the
    device; e2e = wall clock over K further steps (inputs host->device, tokens
    device->host every step)."""
    import torch
    import torch.distributed as dist

    for _ in range(args.warmup):
        eng.step()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    tok0 = sum(s.st.num_output for s in streams)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    n0 = _lib.launch_counter[0]
    for _ in range(args.steps):
        eng.step()
    e1.record()
    barrier()
    launches = _lib.launch_counter[0] - n0
    dev_ms = e0.elapsed_time(e1)
    dev_tokens = sum(s.st.num_output for s in streams) - tok0
    tok1 = sum(s.st.num_output for s in streams)
    h2d0, d2h0 = (mtp.h2d_bytes, mtp.d2h_bytes) if mtp is not None else (eng.h2d_bytes, eng.d2h_bytes)
    t0 = time.perf_counter()
    step_times = []
    for _ in range(args.steps):
        ts = time.perf_counter()
        eng.step()
        step_times.append(time.perf_counter() - ts)
    barrier()
    e2e_s = time.perf_counter() - t0
    e2e_tokens = sum(s.st.num_output for s in streams) - tok1
    if mtp is not None:
        h2d = (mtp.h2d_bytes - h2d0) / args.steps
        d2h = (mtp.d2h_bytes - d2h0) / args.steps
    else:  # eager engine steps: batch inputs host->device, sampled tokens back
        h2d = (eng.h2d_bytes - h2d0) / args.steps
        d2h = (eng.d2h_bytes - d2h0) / args.steps
    clk = clocks.stop()
    t = torch.tensor([dev_ms, e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s = t.tolist()
    st = mtp.stats if mtp is not None else None
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(dev_tokens / (dev_ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random token ids, random-init N(0,0.02) weights; MTP acceptance from a seeded "
                    "Bernoulli(0.7) schedule)",
            "config": {"model": f"{args.model}-shape" + (f" ({cfg.num_layers} layers, DEBUG)" if args.layers else ""),
                       "global_batch": args.streams,
                       "seq_len": f"prompts U[{args.min_prompt},{args.max_prompt}] + {args.out_tokens} out",
                       "parallelism": _par(args, world),
                       "experts": f"q{args.quant_experts} g64" if args.quant_experts else "bf16", "mtp_k": args.mtp,
                       "kv": ("paged fp8-e4m3 (per-head scales)" if args.kv_fp8 else "paged bf16") + ", page 16", "l2": "inputs larger than L2 (weights + KV per step)"},
            "mtp": ({"rounds": st.rounds, "acceptance": round(st.acceptance_rate, 3),
                     "tokens_per_row_round": round(st.emitted / max(st.rows, 1), 3)} if st else None),
            "ttft_p50_ms": round(statistics.median(ttfts) * 1e3, 2),
            "itl_p50_ms": round(statistics.median(step_times) * 1e3, 3), "prefill_s": round(prefill_s, 3),
            "e2e": {"value": round(e2e_tokens / e2e_s, 2), "unit": "tok/s", "api": "EngineV2.step (MTP rounds)",
                    "h2d_bytes_per_step": int(h2d) if h2d is not None else None,
                    "d2h_bytes_per_step": int(d2h) if d2h is not None else None},
            "gpu_launches": int(launches), "clocks": clk, "kernel_status": _lib.read_status(),
        }
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        if getattr(eng.model, "ep", None) is not None:
            eng.model.ep.close()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import numpy as np
    import torch
    import torch.distributed as dist

    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
    from mlx_swift_lm_b200.engine.types import Request, SamplingParams
    from mlx_swift_lm_b200.models import config as mcfg
    from mlx_swift_lm_b200.models.decoder import TensorParallel
    from mlx_swift_lm_b200.ops import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD

    cfg = getattr(mcfg, args.model)()
    if args.layers:
        cfg.num_layers = args.layers
    pp_size = args.pp
    tp_size = world // pp_size
    tp_group = group
    ppc = None
    if pp_size > 1:
        from mlx_swift_lm_b200.parallel.pipeline import PipelineParallel, PipelinedDecoderLM

        stage, tp_rank = rank // tp_size, rank % tp_size
        tp_groups = [dist.new_group(list(range(s * tp_size, (s + 1) * tp_size))) for s in range(pp_size)]
        pp_groups = [dist.new_group([s * tp_size + t for s in range(pp_size)]) for t in range(tp_size)]
        tp_group = tp_groups[stage]
        ppc = PipelineParallel(stage, pp_size, [s * tp_size + tp_rank for s in range(pp_size)], pp_groups[tp_rank])
        tp = TensorParallel(tp_rank, tp_size, tp_group)
        model = PipelinedDecoderLM(cfg, ppc, dev, torch.bfloat16, tp=tp).init_random(args.seed)
    elif args.ep > 1:
        from mlx_swift_lm_b200.parallel.expert import ExpertParallel, ExpertParallelDecoderLM

        assert args.ep == world, "--ep must equal the number of ranks"
        epc = ExpertParallel(cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size, rank, world, group, dev,
                             max_tokens=EP_MAX_TOKENS, impl=args.ep_mode)
        model = ExpertParallelDecoderLM(cfg, epc, dev, torch.bfloat16).init_random(args.seed)
        tp_size = 1
    else:
        tp = TensorParallel(rank, world, group)
        model = DecoderLM(cfg, dev, torch.bfloat16, tp=tp).init_random(args.seed)
    if args.quant_experts or args.quant_dense:
        from mlx_swift_lm_b200.models.quantize import quantize_model

        if args.quant_experts:
            quantize_model(model, bits=args.quant_experts, group_size=64, dense=False, experts=True)
        if args.quant_dense:
            quantize_model(model, bits=args.quant_dense, group_size=64, dense=True, experts=False)
        torch.cuda.empty_cache()
    if tp_size > 1 and args.tp_mode == "fused" and pp_size == 1:
        model.enable_fused_tp(args.streams)
    max_len = args.max_prompt + args.out_tokens + 16
    ecfg = EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=args.streams,
                                                  max_batched_tokens_per_step=EP_MAX_TOKENS if args.ep > 1 else 16384,
                                                  prefill_chunk_size=4096),
                        max_model_len=max_len, use_cuda_graphs=pp_size == 1, chained_decode=True,
                        kv_fp8=args.kv_fp8,
                        graph_buckets=(args.streams,))
    eng = EngineV2(model, config=ecfg)
    mtp = None
    if args.mtp:
        from mlx_swift_lm_b200.engine.mtp import MTPConfig
        from mlx_swift_lm_b200.models.mtp import MTPModule

        mod = MTPModule(model).init_random(args.seed + 1)
        if args.quant_experts:
            from mlx_swift_lm_b200.models.quantize import quantize_model

            quantize_model(mod.inner, bits=args.quant_experts, group_size=64, dense=False, experts=True)
        mtp = eng.enable_mtp(mod, MTPConfig(k=args.mtp, acceptance="bernoulli", p=0.7, seed=args.seed))

    rng = np.random.default_rng(args.seed)
    lens = rng.integers(args.min_prompt, args.max_prompt + 1, size=args.streams)
    prompts = [rng.integers(0, cfg.vocab_size, size=int(n)).tolist() for n in lens]
    greedy = SamplingParams(temperature=0.0)
    streams = [eng.submit(Request(prompt_tokens=p, max_tokens=args.out_tokens, sampling=greedy, ignore_eos=True))
               for p in prompts]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- prefill phase (until every row is decoding) ----
    barrier()
    t_pf = time.perf_counter()
    while any(s.st.timing.first_token == 0 for s in streams):
        eng.step()
    barrier()
    prefill_s = time.perf_counter() - t_pf
    ttfts = [s.st.timing.ttft for s in streams]

    if mtp is not None or pp_size > 1:
        return _mtp_measure(args, eng, mtp, streams, dev, world, rank, ttfts, prefill_s, cfg, barrier, ClockSampler,
                            local, _lib)
    # ---- kernel-only value: replays of the captured decode-step graph ----
    g = eng.graphs
    # one real chained decode step captures/launches the 64-row graph with live inputs
    eng.step()
    eng.step()
    B = g.bucket(args.streams)
    graph = g.graphs[B]
    for _ in range(args.warmup):
        model.begin_step()
        graph.replay()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        model.begin_step()
        graph.replay()
    e1.record()
    barrier()
    dev_ms = e0.elapsed_time(e1)
    launches = args.steps * g.launches_per_replay.get(B, 0)

    # ---- e2e through the public engine API ----
    # the replays above re-wrote the same KV slot; re-run the real step sequence from here
    for _ in range(args.warmup):
        eng.step()
    barrier()
    h2d0, d2h0, n_l0 = g.h2d_bytes, g.d2h_bytes, _lib.launch_counter[0]
    tok0 = sum(s.st.num_output for s in streams)
    t0 = time.perf_counter()
    step_times = []
    for _ in range(args.steps):
        ts = time.perf_counter()
        eng.step()
        step_times.append(time.perf_counter() - ts)
    eng._drain_inflight()
    barrier()
    e2e_s = time.perf_counter() - t0
    clk = clocks.stop()
    tok1 = sum(s.st.num_output for s in streams)
    e2e_tokens = tok1 - tok0
    h2d = (g.h2d_bytes - h2d0) / args.steps
    d2h = (g.d2h_bytes - d2h0) / args.steps
    e2e_launches = _lib.launch_counter[0] - n_l0

    # max over ranks
    t = torch.tensor([dev_ms, e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s = t.tolist()
    ms_per_step = dev_ms / args.steps
    value = args.streams * args.steps / (dev_ms / 1e3)
    e2e_value = e2e_tokens / e2e_s
    itl_p50_ms = statistics.median(step_times) * 1e3
    status = _lib.read_status()
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": (round(value / BASELINE_VALUE, 4) if BASELINE_VALUE else None),
            "dtype": "bf16", "data": "synthetic (random token ids, random-init N(0,0.02) weights)",
            "config": {"model": f"{args.model}-shape" + (f" ({cfg.num_layers} layers, DEBUG)" if args.layers else ""),
                       "global_batch": args.streams, "seq_len": f"prompts U[{args.min_prompt},{args.max_prompt}] + "
                                                                f"{args.out_tokens} out",
                       "parallelism": _par(args, world), "kv": ("paged fp8-e4m3 (per-head scales)" if args.kv_fp8 else "paged bf16") + ", page 16",
                       "l2": "inputs larger than L2 (weights ~16 GB/world + KV per step)"},
            "ttft_p50_ms": round(statistics.median(ttfts) * 1e3, 2),
            "itl_p50_ms": round(itl_p50_ms, 3),
            "prefill_s": round(prefill_s, 3),
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "api": "EngineV2.step (chained CUDA-graph decode)",
                    "gpu_launches": int(e2e_launches)},
            "gpu_launches": int(launches),
            "clocks": clk,
            "kernel_status": status,
        }
        print(json.dumps(out))
    # release every CUDA graph (they may hold NCCL work) and the peer mappings
    # before the process group goes away; otherwise the exit can wait forever
    del graph
    eng.graphs.graphs.clear()
    eng.graphs.pool = None
    import gc

    gc.collect()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
        if getattr(model, "tp_fused", None) is not None:
            model.tp_fused.comm.close()
            model.tp_fused = None
        if getattr(model, "ep", None) is not None:
            model.ep.close()
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
