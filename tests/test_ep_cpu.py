"""Expert parallelism on CPU (gloo): the all-to-all MoE exchange reproduces
the single-rank MoE on every rank's tokens, and a 2-rank expert-parallel
model (data-parallel rows, expert-parallel MoE) generates exactly the tokens
of the whole model."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _moe_cfg():
    c = tiny_qwen3()
    c.num_experts, c.num_experts_per_tok, c.moe_intermediate_size = 8, 2, 128
    c.moe_layers = [True] * c.num_layers
    return c


def _prompts(vocab, lens, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


def _eng(m):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=24),
                                           max_model_len=256, use_cuda_graphs=False))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_pads_to_world():
    from mlx_swift_lm_b200.parallel.expert import shard_rows

    m = DecoderLM(_moe_cfg(), "cpu", torch.float32).init_random(2, std=0.2)
    eng = _eng(m)
    for p in _prompts(m.cfg.vocab_size, (20, 9)):
        eng.submit(__import__("mlx_swift_lm_b200").Request(prompt_tokens=p, max_tokens=4))
    plan = eng.sched.plan()
    fb = eng._build_batch(plan, eng.device)
    parts = shard_rows(fb, 4)
    assert len(parts) == 4
    assert sum(p.num_tokens for p in parts if not p.pad) == fb.num_tokens
    assert [p.pad for p in parts] == [False, False, True, True]


def _ep_worker(rank, world, port, q, seed, prompts):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from mlx_swift_lm_b200.ops import moe as moe_ops
        from mlx_swift_lm_b200.parallel.expert import ExpertParallel, ExpertParallelDecoderLM

        cfg = _moe_cfg()
        # ---- one MoE layer: rank r's tokens through EP == the whole layer
        full = DecoderLM(cfg, "cpu", torch.float32).init_random(seed, std=0.2)
        L = full.layers[0]
        g = torch.Generator().manual_seed(100 + rank)
        T = 5 + 3 * rank
        h = torch.randn(T, cfg.hidden_size, generator=g)
        logits = h @ L.router.t()
        w, idx = moe_ops.route_topk(logits, cfg.num_experts_per_tok)
        want = moe_ops.moe_experts(h, L.experts_gu, L.experts_d, w, idx)
        ep = ExpertParallel(cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size, rank, world,
                            dist.group.WORLD, "cpu")
        got = ep.moe(h, logits, L.experts_gu[ep.lo:ep.hi], L.experts_d[ep.lo:ep.hi])
        layer_err = float((got - want).abs().max())
        # ---- whole model through the engine
        m = ExpertParallelDecoderLM(cfg, ep, "cpu", torch.float32).init_random(seed, std=0.2)
        out = _eng(m).generate(prompts, max_tokens=10)
        # MTP drafting (replicated module) + expert-parallel batched verify
        from mlx_swift_lm_b200.engine.mtp import MTPConfig
        from mlx_swift_lm_b200.models.mtp import MTPModule

        eng = _eng(m)
        drv = eng.enable_mtp(MTPModule(m).init_random(seed + 1, std=0.2), MTPConfig(k=2))
        out_mtp = eng.generate(prompts, max_tokens=10)
        q.put((rank, layer_err, out, m.layers[0].experts_gu.shape[0], out_mtp, drv.stats.rounds))
    finally:
        dist.destroy_process_group()


@pytest.mark.dist
def test_two_rank_expert_parallel_matches_whole_model():
    seed = 4
    m = DecoderLM(_moe_cfg(), "cpu", torch.float32).init_random(seed, std=0.2)
    prompts = _prompts(m.cfg.vocab_size, (17, 40, 6), seed=3)
    ref = _eng(m).generate(prompts, max_tokens=10)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ep_worker, args=(r, 2, port, q, seed, prompts)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(60)
    assert all(p.exitcode == 0 for p in ps)
    for rank, err, out, e_local, out_mtp, rounds in res:
        assert err < 1e-5, (rank, err)
        assert e_local == 4
        assert out == ref, (rank, out, ref)
        assert rounds > 0 and out_mtp == ref, (rank, out_mtp, ref)
