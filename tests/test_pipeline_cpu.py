"""Pipeline parallelism on CPU: microbatch splitting reproduces the full
forward, and a 2-stage gloo pipeline generates exactly the single-model
tokens (last stage samples and broadcasts)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.parallel.pipeline import split_rows, stage_layers


def _prompts(vocab, lens, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


def _eng(m):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=24),
                                           max_model_len=256, use_cuda_graphs=False))


def test_stage_layers_balanced():
    assert stage_layers(80, 2) == [(0, 40), (40, 80)]
    assert stage_layers(10, 4) == [(0, 3), (3, 6), (6, 8), (8, 10)]


def test_split_rows_matches_full_forward():
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(2, std=0.2)
    eng = _eng(m)
    ps = _prompts(m.cfg.vocab_size, (20, 9, 33))
    for p in ps:
        eng.submit(__import__("mlx_swift_lm_b200").Request(prompt_tokens=p, max_tokens=4))
    eng.step()  # prefill chunks of the three rows
    eng.step()
    plan = eng.sched.plan()
    fb = eng._build_batch(plan, eng.device)
    full = m.forward(fb, eng.kv)
    parts = [m.forward(mb, eng.kv) for mb in split_rows(fb, 3)]
    assert len(parts) > 1
    assert torch.allclose(torch.cat(parts, 0), full, atol=1e-4, rtol=1e-5)  # CPU GEMM blocking varies with M


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _pp_worker(rank, world, port, q, seed, prompts):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from mlx_swift_lm_b200.parallel.pipeline import PipelineParallel, PipelinedDecoderLM

        pp = PipelineParallel(rank, world, list(range(world)), dist.group.WORLD)
        m = PipelinedDecoderLM(tiny_qwen3(), pp, "cpu", torch.float32).init_random(seed, std=0.2)
        out = _eng(m).generate(prompts, max_tokens=12)
        q.put((rank, out, len(m.layers)))
    finally:
        dist.destroy_process_group()


@pytest.mark.dist
def test_two_stage_pipeline_matches_single_model():
    seed = 5
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(seed, std=0.2)
    prompts = _prompts(m.cfg.vocab_size, (17, 40, 6), seed=3)
    ref = _eng(m).generate(prompts, max_tokens=12)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_pp_worker, args=(r, 2, port, q, seed, prompts)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in ps:
        p.join(60)
    assert all(p.exitcode == 0 for p in ps)
    for rank, out, nl in res:
        assert nl == 2
        assert out == ref, (rank, out, ref)
