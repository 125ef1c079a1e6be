#!/usr/bin/env python3
"""Headline benchmark: decode tok/s at 64 concurrent streams (+ p50 TTFT / ITL).

Config (benchmark config 2): Qwen3-8B-shape dense decoder, bf16, random-init
N(0, 0.02) weights, paged KV (page 16), 64 requests with prompt lengths
uniform in [128, 2048] (random token ids), 256 output tokens each, greedy.
Tensor parallel over all GPUs of the run (tp = N).

Measurement (per arm):
  * prefill phase: all 64 requests are submitted and the engine steps until
    every row decodes; TTFT p50 comes from the engine's per-request timing.
  * ``value``: W warm-up engine steps, then K consecutive decode steps through
    ``EngineV2.step`` (chained CUDA-graph decode of the 64 rows at their live
    KV positions), bracketed by CUDA events on the launching stream with a
    barrier + synchronize on both sides; max over ranks. Inputs (weights
    16 GB / N + KV) exceed L2.
  * ``e2e``: wall clock from the first timed step until every request has all
    its output tokens, through the same public API; every step copies its
    inputs host->device from pinned memory and reads its tokens back. ITL p50
    is the median engine step over that window.

Arms: ``--impl ours`` runs the framework, then (dense bf16 configurations)
the NCCL+cuBLAS arm of the same model, engine and workload in the same
process, and reports ``vs_baseline`` = value / that arm's value.
``--impl baseline`` runs only that arm; ``--impl reference`` reports that the
upstream project cannot run here.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|baseline|reference]
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "baseline", "reference"],
                    help="ours: the framework; baseline: the same engine with PyTorch/cuBLAS/NCCL ops only; "
                         "reference: the upstream project (unavailable here)")
    ap.add_argument("--diag", action="store_true",
                    help="diagnostic: replay the full-batch decode graph after the warm-up and report its time")
    ap.add_argument("--timeline", default="",
                    help="diagnostic: write the device timeline of one decode-graph replay to this path "
                         "({rank} is replaced by the rank)")
    ap.add_argument("--no-compare", dest="compare", action="store_false",
                    help="skip the NCCL+cuBLAS arm that --impl ours runs after itself for vs_baseline")
    ap.add_argument("--model", default="qwen3_8b")
    ap.add_argument("--streams", type=int, default=64)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=2048)
    ap.add_argument("--out-tokens", type=int, default=256)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (debug only; invalid for the headline)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--temperature", type=float, default=0.0, help="sampled traffic (0 = greedy)")
    ap.add_argument("--top-p", type=float, default=1.0)
    ap.add_argument("--tp-mode", default=None, choices=["fused", "nccl"],
                    help="tensor-parallel collectives: fused symmetric-memory kernels (default with 2+ GPUs) or "
                         "NCCL all-reduce")
    ap.add_argument("--quant-experts", type=int, default=0, help="MLX affine bits for MoE experts (0 = bf16)")
    ap.add_argument("--expert-format", default="affine", choices=["affine", "mxfp4"],
                    help="quantised expert records: MLX affine (group 64) or MXFP4 (e2m1 + e8m0 per 32, GPT-OSS)")
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


def receipt(dev) -> dict:
    """Provenance of a run (the reference's bench receipts: revision stamp,
    hardware, software): a hash of the framework's sources (the snapshot that
    ran, with or without git), the GPU SKU, driver, CUDA / torch / NCCL
    versions."""
    import hashlib

    import torch

    h = hashlib.sha256()
    pkg = os.path.join(ROOT, "mlx_swift_lm_b200")
    for d, _, files in sorted(os.walk(pkg)):
        if "_lib" in d or "__pycache__" in d:
            continue
        for f in sorted(files):
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
    with open(os.path.abspath(__file__), "rb") as fh:
        h.update(fh.read())
    drv = None
    try:
        drv = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=10).stdout.strip().splitlines()[0]
    except Exception:
        pass
    props = torch.cuda.get_device_properties(dev)
    nccl = None
    try:
        nccl = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception:
        pass
    return {"source_sha256": h.hexdigest()[:16], "gpu": props.name, "sm": f"{props.major}{props.minor}",
            "sms": props.multi_processor_count, "hbm_gb": round(props.total_memory / 1e9, 1), "driver": drv,
            "cuda": torch.version.cuda, "torch": torch.__version__, "nccl": nccl}


def _release(eng, model, world):
    """Drop graphs (they may hold NCCL work), peer mappings and the model's
    memory so the next arm starts from a clean device."""
    import gc

    import torch

    eng.release_graphs()
    if getattr(model, "tp_fused", None) is not None:
        model.tp_fused.comm.close()
        model.tp_fused = None
    if getattr(model, "ep", None) is not None:
        model.ep.close()
    gc.collect()
    torch.cuda.synchronize(eng.device)
    torch.cuda.empty_cache()


def _build(args, impl, world, rank, dev, group):
    """(model, engine, mtp driver or None) of one arm."""
    import torch
    import torch.distributed as dist

    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
    from mlx_swift_lm_b200.models import config as mcfg
    from mlx_swift_lm_b200.models.decoder import TensorParallel

    cfg = getattr(mcfg, args.model)()
    if args.layers:
        cfg.num_layers = args.layers
    pp_size = args.pp
    tp_size = world // pp_size
    if impl == "baseline":
        from mlx_swift_lm_b200.baseline import TorchDecoderLM

        if pp_size > 1 or args.ep > 1 or args.mtp or args.quant_experts or args.quant_dense or args.kv_fp8:
            raise ValueError("the NCCL+cuBLAS baseline arm runs the dense bf16 TP configuration only")
        model = TorchDecoderLM(cfg, dev, torch.bfloat16, tp=TensorParallel(rank, world, group)).init_random(args.seed)
    elif pp_size > 1:
        from mlx_swift_lm_b200.parallel.pipeline import PipelineParallel, PipelinedDecoderLM

        stage, tp_rank = rank // tp_size, rank % tp_size
        tp_groups = [dist.new_group(list(range(s * tp_size, (s + 1) * tp_size))) for s in range(pp_size)]
        pp_groups = [dist.new_group([s * tp_size + t for s in range(pp_size)]) for t in range(tp_size)]
        ppc = PipelineParallel(stage, pp_size, [s * tp_size + tp_rank for s in range(pp_size)], pp_groups[tp_rank])
        tp = TensorParallel(tp_rank, tp_size, tp_groups[stage])
        model = PipelinedDecoderLM(cfg, ppc, dev, torch.bfloat16, tp=tp).init_random(args.seed)
    elif args.ep > 1:
        from mlx_swift_lm_b200.parallel.expert import ExpertParallel, ExpertParallelDecoderLM

        assert args.ep == world, "--ep must equal the number of ranks"
        epc = ExpertParallel(cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size, rank, world, group, dev,
                             max_tokens=EP_MAX_TOKENS, impl=args.ep_mode)
        model = ExpertParallelDecoderLM(cfg, epc, dev, torch.bfloat16).init_random(args.seed)
        tp_size = 1
    else:
        hook = None
        if impl == "ours" and args.quant_experts:
            # quantise each layer's experts as it is drawn: the bf16 experts of
            # a GPT-OSS-120B-shaped model alone would not fit on one device
            from mlx_swift_lm_b200.models.quantize import quantize_layer

            def hook(L):
                return quantize_layer(L, dev, bits=args.quant_experts, group_size=64, dense=False, experts=True,
                                      mode=args.expert_format)
        model = DecoderLM(cfg, dev, torch.bfloat16, tp=TensorParallel(rank, world, group)).init_random(
            args.seed, layer_hook=hook)
    if impl == "ours" and (args.quant_experts or args.quant_dense):
        from mlx_swift_lm_b200.models.quantize import quantize_model

        if args.quant_experts:  # no-op for layers the init hook already quantised
            quantize_model(model, bits=args.quant_experts, group_size=64, dense=False, experts=True,
                           mode=args.expert_format)
        if args.quant_dense:
            quantize_model(model, bits=args.quant_dense, group_size=64, dense=True, experts=False)
        torch.cuda.empty_cache()
    if impl == "ours" and tp_size > 1 and args.tp_mode == "fused" and pp_size == 1:
        model.enable_fused_tp(args.streams)
    max_len = args.max_prompt + args.out_tokens + 16
    ecfg = EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=args.streams,
                                                  max_batched_tokens_per_step=EP_MAX_TOKENS if args.ep > 1 else 16384,
                                                  prefill_chunk_size=4096),
                        max_model_len=max_len, use_cuda_graphs=pp_size == 1, chained_decode=True,
                        kv_fp8=args.kv_fp8, graph_buckets=(args.streams,))
    eng = EngineV2(model, config=ecfg)
    if impl == "baseline":
        model.bind_engine(eng)
    mtp = None
    if args.mtp:
        from mlx_swift_lm_b200.engine.mtp import MTPConfig
        from mlx_swift_lm_b200.models.mtp import MTPModule

        mod = MTPModule(model).init_random(args.seed + 1)
        if args.quant_experts:
            from mlx_swift_lm_b200.models.quantize import quantize_model

            quantize_model(mod.inner, bits=args.quant_experts, group_size=64, dense=False, experts=True)
        mtp = eng.enable_mtp(mod, MTPConfig(k=args.mtp, acceptance="bernoulli", p=0.7, seed=args.seed))
    return cfg, model, eng, mtp


def run_arm(args, impl, world, rank, local, dev, group):
    """One measured arm: submit the 64 requests, prefill until every row
    decodes (TTFT), W warm-up engine steps, then K engine steps timed on the
    device (CUDA events on the launching stream, max over ranks) for `value`,
    and the wall clock from the first timed step until every request has
    produced all its tokens for `e2e` (every step copies its inputs
    host->device from pinned memory and reads its tokens back)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from mlx_swift_lm_b200.engine.scheduler import Status
    from mlx_swift_lm_b200.engine.types import Request, SamplingParams
    from mlx_swift_lm_b200.ops import _lib

    cfg, model, eng, mtp = _build(args, impl, world, rank, dev, group)
    # untimed warm-up request: first-use costs (lazy module loads, library
    # initialisation, first graph captures of small buckets) stay out of TTFT
    warm = [eng.submit(Request(prompt_tokens=list(range(1, 65 + 31 * i)), max_tokens=4,
                               sampling=SamplingParams(temperature=0.0), ignore_eos=True)) for i in range(2)]
    while any(s.st.status != Status.FINISHED for s in warm):
        eng.step()
    eng._drain_inflight()
    if world > 1:
        dist.barrier()
    rng = np.random.default_rng(args.seed)
    lens = rng.integers(args.min_prompt, args.max_prompt + 1, size=args.streams)
    prompts = [rng.integers(0, cfg.vocab_size, size=int(n)).tolist() for n in lens]
    def sp(i):
        if args.temperature <= 0:
            return SamplingParams(temperature=0.0)
        return SamplingParams(temperature=args.temperature, top_p=args.top_p, seed=args.seed * 1000 + i)

    streams = [eng.submit(Request(prompt_tokens=p, max_tokens=args.out_tokens, sampling=sp(i), ignore_eos=True))
               for i, p in enumerate(prompts)]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def emitted():
        return sum(s.st.num_output for s in streams)

    def moved():
        g = eng.graphs
        h = eng.h2d_bytes + (g.h2d_bytes if g is not None else 0) + (mtp.h2d_bytes if mtp is not None else 0)
        d = eng.d2h_bytes + (g.d2h_bytes if g is not None else 0) + (mtp.d2h_bytes if mtp is not None else 0)
        return h, d

    # ---- prefill phase (until every row is decoding) ----
    barrier()
    t_pf = time.perf_counter()
    while any(s.st.timing.first_token == 0 for s in streams):
        eng.step()
    barrier()
    prefill_s = time.perf_counter() - t_pf
    ttfts = [s.st.timing.ttft for s in streams]
    assert args.warmup + args.steps + 2 < args.out_tokens, "timed steps must end before the first request finishes"

    for _ in range(args.warmup):
        eng.step()
    barrier()
    # diagnostic (opt-in, --diag / --timeline): the decode graph of the full batch
    # replayed back to back after the warm-up (device time of one step with no host
    # work between replays; it rewrites the K/V of the last step's positions)
    replay_ms = None
    g = eng.graphs
    runner = getattr(mtp, "runner", None) if mtp is not None else None
    if (args.diag or args.timeline) and runner is not None and impl == "ours":
        # MTP: the captured round of the full batch instead of a decode graph
        R = next((R for (B, k), R in sorted(runner.rounds.items()) if B >= args.streams and R.graph is not None),
                 None)
        if R is not None:
            eng._drain_inflight()
            barrier()
            r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            r0.record()
            for _ in range(10):
                model.begin_step()
                R.graph.replay()
            r1.record()
            barrier()
            replay_ms = round(r0.elapsed_time(r1) / 10, 4)
            if args.timeline:
                from mlx_swift_lm_b200.engine.diagnostics import timeline_summary

                tl = _lib.timeline_start(dev)
                model.begin_step()
                R.graph.replay()
                torch.cuda.synchronize(dev)
                marks = _lib.timeline_read(tl)
                _lib.timeline_stop()
                with open(args.timeline.replace("{rank}", str(rank)), "w") as f:
                    f.write(timeline_summary(marks, f"MTP round graph replay (B={R.B}, k={R.k}), rank {rank}") + "\n")
    elif (args.diag or args.timeline) and g is not None and args.streams in g.graphs:
        eng._drain_inflight()
        barrier()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for _ in range(20):
            model.begin_step()
            g.graphs[args.streams].replay()
        r1.record()
        barrier()
        rt = torch.tensor([r0.elapsed_time(r1) / 20], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(rt, op=dist.ReduceOp.MAX)
        replay_ms = round(rt.item(), 4)
        if args.timeline and impl == "ours":
            from mlx_swift_lm_b200.engine.diagnostics import timeline_summary

            tl = _lib.timeline_start(dev)
            model.begin_step()
            g.graphs[args.streams].replay()
            torch.cuda.synchronize(dev)
            marks = _lib.timeline_read(tl)
            _lib.timeline_stop()
            with open(args.timeline.replace("{rank}", str(rank)), "w") as f:
                f.write(timeline_summary(marks, f"decode graph replay, rank {rank} of {world}, "
                                                f"{args.streams} rows") + "\n")
            barrier()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tok0 = emitted()
    h0, d0 = moved()
    n_l0 = _lib.launch_counter[0]
    step_times = []
    t0 = time.perf_counter()
    e0.record()
    for _ in range(args.steps):
        ts = time.perf_counter()
        eng.step()
        step_times.append(time.perf_counter() - ts)
    e1.record()
    launches = _lib.launch_counter[0] - n_l0
    tok_timed = emitted() - tok0
    # ---- the rest of the decode, to the last token of every request ----
    n_steps = args.steps
    while any(s.st.status != Status.FINISHED for s in streams):
        ts = time.perf_counter()
        eng.step()
        step_times.append(time.perf_counter() - ts)
        n_steps += 1
    eng._drain_inflight()
    barrier()
    e2e_s = time.perf_counter() - t0
    clk = clocks.stop()
    dev_ms = e0.elapsed_time(e1)
    e2e_tokens = emitted() - tok0
    h1, d1 = moved()
    t = torch.tensor([dev_ms, e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s = t.tolist()
    st = mtp.stats if mtp is not None else None
    res = {
        "diag": {"graph_replay_ms": replay_ms, "host_step_ms_p50": round(statistics.median(step_times) * 1e3, 3),
                 "step_kinds": dict(eng.step_kinds)},
        "value": round(tok_timed / (dev_ms / 1e3), 2), "ms_per_step": round(dev_ms / args.steps, 4),
        "ttft_p50_ms": round(statistics.median(ttfts) * 1e3, 2),
        "itl_p50_ms": round(statistics.median(step_times) * 1e3, 3), "prefill_s": round(prefill_s, 3),
        "e2e": {"value": round(e2e_tokens / e2e_s, 2), "unit": "tok/s",
                "h2d_bytes_per_step": int((h1 - h0) / n_steps), "d2h_bytes_per_step": int((d1 - d0) / n_steps),
                "api": "EngineV2.step" + (" (MTP rounds)" if mtp is not None else " (chained CUDA-graph decode)"),
                "window": f"{n_steps} engine steps: the {args.steps} device-timed steps, then every step until all "
                          f"{args.streams} requests have their {args.out_tokens} tokens"},
        "gpu_launches": int(launches), "clocks": clk, "cfg": cfg,
        "mtp": ({"rounds": st.rounds, "acceptance": round(st.acceptance_rate, 3),
                 "tokens_per_row_round": round(st.emitted / max(st.rows, 1), 3)} if st else None),
        "kernel_status": _lib.read_status(),
    }
    _release(eng, model, world)
    del eng, model
    return res


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import gc

    import torch
    import torch.distributed as dist

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
    if args.tp_mode is None:
        args.tp_mode = "fused" if world > 1 else "nccl"

    res = run_arm(args, args.impl, world, rank, local, dev, group)
    base, why = None, None
    dense = not (args.pp > 1 or args.ep > 1 or args.mtp or args.quant_experts or args.quant_dense or args.kv_fp8
                 or args.temperature > 0)
    if args.impl == "ours" and args.compare and dense:
        gc.collect()
        base = run_arm(args, "baseline", world, rank, local, dev, group)
    elif args.impl == "ours":
        why = ("no NCCL+cuBLAS arm for this configuration (dense bf16 greedy TP only)" if not dense
               else "--no-compare")
    cfg = res.pop("cfg")
    if rank == 0:
        out = {"metric": METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
               "scaling": "strong"}
        if args.impl != "ours":
            out["impl"] = args.impl
        out["vs_baseline"] = round(res["value"] / base["value"], 4) if base else None
        out.update({
            "dtype": "bf16",
            "data": "synthetic (random token ids, random-init N(0,0.02) weights"
                    + ("; MTP acceptance from a seeded Bernoulli(0.7) schedule)" if args.mtp else ")"),
            "config": {"model": f"{args.model}-shape" + (f" ({cfg.num_layers} layers, DEBUG)" if args.layers else ""),
                       "global_batch": args.streams,
                       "seq_len": f"prompts U[{args.min_prompt},{args.max_prompt}] + {args.out_tokens} out",
                       "parallelism": _par(args, world) if args.impl == "ours" else f"tp{world} (NCCL all_reduce)",
                       "experts": ("mxfp4 g32" if args.expert_format == "mxfp4" else f"q{args.quant_experts} g64")
                       if args.quant_experts else "bf16", "mtp_k": args.mtp,
                       "kv": ("paged fp8-e4m3 (per-head scales)" if args.kv_fp8 else "paged bf16") + ", page 16",
                       "sampling": ("greedy" if args.temperature <= 0 else
                                    f"temperature {args.temperature}, top_p {args.top_p}, per-request seeds"),
                       "l2": "inputs larger than L2 (weights ~16 GB/world + KV per step)",
                       "timed": f"value: {args.steps} consecutive engine decode steps (64 rows, live KV positions) "
                                f"after {args.warmup} warm-up steps, CUDA events, max over ranks"},
        })
        for k in ("ttft_p50_ms", "itl_p50_ms", "prefill_s", "e2e", "gpu_launches", "clocks", "mtp", "kernel_status",
                  "diag"):
            out[k] = res[k]
        out["receipt"] = receipt(dev)
        if base is not None:
            out["baseline"] = {"impl": "PyTorch: cuBLAS GEMMs (F.linear), SDPA over gathered pages, NCCL all_reduce, "
                                       "same engine and CUDA-graph decode",
                               "value": base["value"], "ms_per_step": base["ms_per_step"],
                               "ttft_p50_ms": base["ttft_p50_ms"], "itl_p50_ms": base["itl_p50_ms"],
                               "e2e": base["e2e"]["value"], "clocks": base["clocks"]}
            out["vs_baseline_e2e"] = round(res["e2e"]["value"] / base["e2e"]["value"], 4)
        elif why:
            out["baseline"] = {"unavailable": why}
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
