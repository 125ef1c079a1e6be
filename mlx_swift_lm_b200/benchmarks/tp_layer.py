"""Tensor-parallel decode collectives of one Qwen3-8B layer, fused vs NCCL:
per-primitive device time at M decode rows, max over ranks, against the
primitive's roofline.

    timeout -k 60 600 torchrun --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m mlx_swift_lm_b200.benchmarks.tp_layer [--rows 64] [--layers 4]

Fused primitives (parallel/tp_fused.py): AG->GEMM (qkv, gate/up: every rank
reads the gathered rows of all ranks' normalised hidden state from symmetric
memory inside the GEMM prologue), GEMM->RS (o_proj, down: fp32 partial rows
stored into the owner rank's inbox from the GEMM epilogue) and the
combine-norm that sums the inboxes, adds the residual, normalises and
publishes. Baseline: ops.gemm on the full rows plus NCCL all_gather /
reduce_scatter of the same tensors.

Roofline of a primitive = max(weight bytes / HBM bandwidth, FLOPs / bf16
peak, NVLink bytes / 770 GB/s per direction) with the pool's measured peaks
(``MEASURED_PEAKS.json`` at the repository root when present, else 6.65 TB/s
and 1.59 PFLOP/s).
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

LINK = 770e9


def _peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]) * 1e9, float(d["bf16_tflops"]) * 1e12, "measured"
    except Exception:
        return 6.65e12, 1.59e15, "fallback"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--reps", type=int, default=50)
    a = ap.parse_args(argv)
    from ..models import config as mcfg
    from ..models.decoder import DecoderLM, TensorParallel
    from ..ops import _lib
    from .. import ops

    world, rank, local = (int(os.environ[k]) for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cfg = mcfg.qwen3_8b()
    cfg.num_layers = a.layers
    m = DecoderLM(cfg, dev, torch.bfloat16, tp=TensorParallel(rank, world, dist.group.WORLD)).init_random(0)
    m.enable_fused_tp(a.rows)
    ft = m.tp_fused
    T, Hd = a.rows, cfg.hidden_size
    ids = torch.randint(0, cfg.vocab_size, (T,), device=dev, dtype=torch.int32)
    attn = torch.randn(T, m.H * m.D, device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    st = _lib.stream_ptr(dev)
    names = ["ag_qkv", "rs_o", "norm1", "ag_gu", "rs_down", "norm2"]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    acc = {n: 0.0 for n in names}

    def fused_pass(timed):
        ft.comm.phase = 0
        _lib.check(L.b200_tp_embed(ft.comm.ctx_ptr, ids.data_ptr(), T, m.embed.data_ptr(), m.embed.shape[0],
                                   ft.x_local.data_ptr(), 1.0, st), "tp_embed")
        ag = ft._publish(m.layers[0].ln1, False, None)
        for li, Lw in enumerate(m.layers):
            if timed:
                ev[0].record()
            ft._gemm_ag(ag, T, Lw.wqkv, ft.qkv, bias=Lw.bqkv)
            if timed:
                ev[1].record()
            rs = ft._gemm_rs(attn, T, Lw.wo, Lw.bo)
            if timed:
                ev[2].record()
            ag = ft._publish(Lw.ln2, True, rs)
            if timed:
                ev[3].record()
            ft._gemm_ag(ag, T, Lw.wgu, ft.gu, epi=cfg.glu_epi, bias=Lw.bgu)
            if timed:
                ev[4].record()
            rs = ft._gemm_rs(ft.gu[:T], T, Lw.wd, Lw.bd)
            if timed:
                ev[5].record()
            nxt = m.layers[li + 1].ln1 if li + 1 < len(m.layers) else m.norm
            ag = ft._publish(nxt, True, rs)
            if timed:
                ev[6].record()
                torch.cuda.synchronize()
                for i, n in enumerate(names):
                    acc[n] += ev[i].elapsed_time(ev[i + 1]) * 1e3

    # NCCL baseline: the same GEMMs on full rows + all_gather / reduce_scatter
    rpr = ft.rpr
    h_loc = torch.randn(rpr, Hd, device=dev, dtype=torch.bfloat16)
    h_all = torch.empty(world * rpr, Hd, device=dev, dtype=torch.bfloat16)
    base = {n: 0.0 for n in ("ag+gemm_qkv", "gemm+rs_o", "ag+gemm_gu", "gemm+rs_down")}

    def nccl_pass(timed):
        for Lw in m.layers:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            e[0].record()
            dist.all_gather_into_tensor(h_all, h_loc)
            ops.gemm(h_all[:T], Lw.wqkv, bias=Lw.bqkv)
            e[1].record()
            y = ops.gemm(attn, Lw.wo, epi="f32")
            out = torch.empty(T // world, y.shape[1], device=dev, dtype=torch.float32)
            dist.reduce_scatter_tensor(out, y[:out.shape[0] * world])
            e[2].record()
            dist.all_gather_into_tensor(h_all, h_loc)
            gu = ops.gemm(h_all[:T], Lw.wgu, epi=cfg.glu_epi, bias=Lw.bgu)
            e[3].record()
            y = ops.gemm(gu, Lw.wd, epi="f32")
            dist.reduce_scatter_tensor(out, y[:out.shape[0] * world])
            e[4].record()
            if timed:
                torch.cuda.synchronize()
                for i, n in enumerate(base):
                    base[n] += e[i].elapsed_time(e[i + 1]) * 1e3

    for fn, res in ((fused_pass, acc), (nccl_pass, base)):
        for _ in range(5):
            fn(False)
        torch.cuda.synchronize()
        dist.barrier()
        for _ in range(a.reps):
            fn(True)
        for n in res:
            res[n] /= a.reps * a.layers
    # max over ranks
    vals = torch.tensor([acc[n] for n in names] + [base[n] for n in base], device=dev)
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    v = vals.tolist()
    if rank == 0:
        hbm, flops, src = _peaks()
        K, D = Hd, m.D
        Nqkv = (m.H + 2 * m.KVH) * D  # rank-local rows
        Ngu, F = m.layers[0].wgu.shape[0], m.layers[0].wd.shape[1]

        def roof(wbytes, fl, link):
            return max(wbytes / hbm, fl / flops, link / LINK) * 1e6

        rows = {
            "ag_qkv": roof(Nqkv * K * 2, 2 * T * Nqkv * K, (world - 1) * rpr * K * 2),
            "rs_o": roof(K * m.H * D * 2, 2 * T * K * m.H * D, (world - 1) * rpr * K * 4),
            "ag_gu": roof(Ngu * K * 2, 2 * T * Ngu * K, (world - 1) * rpr * K * 2),
            "rs_down": roof(K * F * 2, 2 * T * K * F, (world - 1) * rpr * K * 4),
        }
        print(f"qwen3-8b layer, TP={world}, M={T} decode rows, peaks: {src} "
              f"({hbm / 1e12:.2f} TB/s, {flops / 1e15:.2f} PFLOP/s, link 770 GB/s)")
        for i, n in enumerate(names):
            r = rows.get(n)
            frac = f"  roofline {r:6.1f} us  achieved/roofline {r / v[i]:.2f}" if r else ""
            print(f"  fused {n:8s} {v[i]:7.1f} us{frac}")
        for j, n in enumerate(base):
            print(f"  nccl  {n:13s} {v[len(names) + j]:7.1f} us")
        tot_f = sum(v[:len(names)])
        tot_b = sum(v[len(names):])
        print(f"  per layer: fused {tot_f:.1f} us (incl. 2 combine-norms), nccl {tot_b:.1f} us (norms excluded)")
    m.tp_fused.comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
