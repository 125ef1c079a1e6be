"""Expert-parallel kernels (fused router top-k + dispatch over symmetric
memory, owner-side prepare / return, weighted combine) against the
single-rank MoE, on one GPU (the rank dispatches to itself) and, where the box
has two GPUs, across two ranks against the all-to-all baseline and the whole
model."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mlx_swift_lm_b200.ops import moe
from mlx_swift_lm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _experts(E, K, F, seed, bits=0):
    from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

    g = torch.Generator().manual_seed(seed)
    gu = [ref.interleave_gate_up(torch.randn(F, K, generator=g) * 0.05, torch.randn(F, K, generator=g) * 0.05)
          for _ in range(E)]
    d = [torch.randn(K, F, generator=g) * 0.05 for _ in range(E)]
    if bits:
        return (QuantizedWeight.stack_experts([QuantizedWeight.quantize(t, bits, 64) for t in gu]).to(DEV),
                QuantizedWeight.stack_experts([QuantizedWeight.quantize(t, bits, 64) for t in d]).to(DEV))
    return (torch.stack(gu).to(DEV, torch.bfloat16), torch.stack(d).to(DEV, torch.bfloat16))


@pytest.mark.parametrize("bits", [0, 4])
@pytest.mark.parametrize("T,E,k", [(1, 16, 4), (64, 16, 4), (300, 32, 8)])
def test_ep_fused_single_rank_matches_moe(T, E, k, bits):
    from mlx_swift_lm_b200.ops import _lib
    from mlx_swift_lm_b200.parallel.expert import ExpertParallel

    K, F = 512, 256
    gu, d = _experts(E, K, F, seed=T + E, bits=bits)
    ep = ExpertParallel(E, k, K, 0, 1, None, DEV, max_tokens=2 * T + 4)
    assert ep.impl == "fused"
    torch.manual_seed(T)
    for it in range(3):
        h = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
        lg = torch.randn(T, E, device=DEV)
        w, idx = moe.route_topk(lg, k)
        want = moe.moe_experts(h, gu, d, w, idx)
        ep.begin_step()
        got = ep.moe(h, lg, gu, d, tokens_max=T + it)  # capacity above this rank's tokens
        torch.cuda.synchronize()
        assert _lib.read_status().get("ep", 0) == 0
        assert _rel(got, want) < 1e-3, it
    ep.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tiny_moe_cfg():
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    c = tiny_qwen3()
    c.model_type = "qwen3_moe"
    c.num_experts, c.num_experts_per_tok, c.moe_intermediate_size = 16, 4, 128
    c.moe_layers = [True] * c.num_layers
    return c


def _worker(rank, world, port, q, prompts):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from mlx_swift_lm_b200 import EngineConfig, EngineV2, SchedulerConfig
        from mlx_swift_lm_b200.ops import _lib
        from mlx_swift_lm_b200.parallel.expert import ExpertParallel, ExpertParallelDecoderLM

        E, k, K, F = 32, 8, 512, 256
        g = torch.Generator().manual_seed(7)
        gu = torch.stack([ref.interleave_gate_up(torch.randn(F, K, generator=g) * 0.05,
                                                 torch.randn(F, K, generator=g) * 0.05) for _ in range(E)])
        d = torch.stack([torch.randn(K, F, generator=g) * 0.05 for _ in range(E)])
        gu, d = gu.to(dev, torch.bfloat16), d.to(dev, torch.bfloat16)
        fused = ExpertParallel(E, k, K, rank, world, dist.group.WORLD, dev, max_tokens=128)
        a2a = ExpertParallel(E, k, K, rank, world, dist.group.WORLD, dev, max_tokens=128, impl="a2a")
        errs = []
        for it in range(3):
            T = 40 + 30 * rank + it
            h = torch.randn(T, K, device=dev, dtype=torch.bfloat16, generator=torch.Generator(dev).manual_seed(it))
            lg = torch.randn(T, E, device=dev, generator=torch.Generator(dev).manual_seed(50 + it + rank))
            w, idx = moe.route_topk(lg, k)
            want = moe.moe_experts(h, gu, d, w, idx)
            fused.begin_step()
            y1 = fused.moe(h, lg, gu[fused.lo:fused.hi], d[fused.lo:fused.hi], tokens_max=72 + it)
            y2 = a2a.moe(h, lg, gu[a2a.lo:a2a.hi], d[a2a.lo:a2a.hi])
            torch.cuda.synchronize()
            errs.append((_rel(y1, want), _rel(y2, want)))
        status = _lib.read_status().get("ep", 0)
        fused.close()
        # whole model: expert-parallel engine (graphs and eager) on every rank
        cfg = _tiny_moe_cfg()
        ep = ExpertParallel(cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size, rank, world,
                            dist.group.WORLD, dev, max_tokens=256)
        m = ExpertParallelDecoderLM(cfg, ep, dev, torch.bfloat16).init_random(3, std=0.2)
        outs = []
        for graphs in (True, False):
            eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4,
                                                                            prefill_chunk_size=64),
                                                  max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(2, 4)))
            outs.append(eng.generate(prompts, max_tokens=12))
            eng.release_graphs()  # graphs hold NCCL calls: release before the group goes
            del eng
        torch.cuda.synchronize()
        status |= _lib.read_status().get("ep", 0)
        ep.close()
        q.put((rank, errs, status, outs))
    finally:
        dist.destroy_process_group()


@pytest.mark.dist
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_ranks():
    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig

    g = torch.Generator().manual_seed(11)
    cfg = _tiny_moe_cfg()
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 77)]
    whole = DecoderLM(cfg, DEV, torch.bfloat16).init_random(3, std=0.2)
    ref_out = EngineV2(whole, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4,
                                                                            prefill_chunk_size=64),
                                                  max_model_len=256, use_cuda_graphs=False)).generate(
        prompts, max_tokens=12)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, prompts)) for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = [q.get(timeout=300) for _ in range(2)]
    finally:
        for p in ps:
            p.join(60)
            if p.is_alive():
                p.kill()
                p.join(10)
    for rank, errs, status, outs in res:
        print(rank, errs, status)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for rank, errs, status, outs in res:
        assert status == 0, (rank, status)
        for e1, e2 in errs:
            assert e1 < 1e-3 and e2 < 1e-3, (rank, errs)
        assert outs[0] == outs[1], (rank, outs)
        assert outs[1] == ref_out, (rank, outs[1], ref_out)
