"""Tensor parallelism on 2 GPUs: the fused symmetric-memory decode path and
the NCCL path produce the single-GPU tokens. Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.dist]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(wide):
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    c = tiny_qwen3()
    if wide:  # heads, KV-head replication and MLP shards that split 8 ways
        c.hidden_size, c.num_heads, c.num_kv_heads, c.head_dim, c.intermediate_size = 512, 8, 2, 64, 1024
    return c


def _worker(rank, world, port, mode, q, wide=False, nvls=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      B200LM_TP_NVLS="1" if nvls else "0")
    from datetime import timedelta

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
        from mlx_swift_lm_b200.models.config import tiny_qwen3
        from mlx_swift_lm_b200.models.decoder import TensorParallel

        cfg = _cfg(wide)
        m = DecoderLM(cfg, dev, torch.bfloat16, tp=TensorParallel(rank, world, dist.group.WORLD)).init_random(
            5, std=0.2)
        ok, nvls_on = True, False
        if mode == "fused":
            m.enable_fused_tp(8)
            ok = m.tp_fused.comm.self_test()
            nvls_on = m.tp_fused.rs_mode == 3
        eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=8),
                                              max_model_len=256, graph_buckets=(1, 2, 4, 8)))
        g = torch.Generator().manual_seed(1)
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 7, 33)]
        out = eng.generate(prompts, max_tokens=12)
        from mlx_swift_lm_b200.ops import _lib

        st = _lib.read_status()
        if rank == 0:
            q.put((out, ok, st, nvls_on))
        # graphs may hold NCCL work and peer addresses: release them, then the
        # peer mappings, before the process group goes away
        if eng.graphs is not None:
            eng.graphs.graphs.clear()
            eng.graphs.pool = None
        import gc

        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        if m.tp_fused is not None:
            m.tp_fused.comm.close()
            m.tp_fused = None  # drops the multicast-bound buffer too
            gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(mode, world=2, wide=False, nvls=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q, wide, nvls)) for r in range(world)]
    for p in ps:
        p.start()
    res = q.get(timeout=600)
    for p in ps:
        p.join(120)
    assert all(p.exitcode == 0 for p in ps)
    return res[:3] if not nvls else res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_fused_and_nccl_match_single_gpu():
    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    cfg = tiny_qwen3()
    m = DecoderLM(cfg, torch.device("cuda", 0), torch.bfloat16).init_random(5, std=0.2)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=8), max_model_len=256,
                                          graph_buckets=(1, 2, 4, 8)))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 7, 33)]
    ref = eng.generate(prompts, max_tokens=12)
    fused, ok, st = _run("fused")
    assert ok, "symmetric-memory signal round trip failed"
    assert all(v == 0 for v in st.values()), st
    nccl, _, _ = _run("nccl")
    agree_f = sum(a == b for x, y in zip(fused, ref) for a, b in zip(x, y)) / 36
    agree_n = sum(a == b for x, y in zip(nccl, ref) for a, b in zip(x, y)) / 36
    assert agree_f >= 0.75 and agree_n >= 0.75, (fused, nccl, ref)


@pytest.mark.parametrize("world", [4, 8])
def test_tp_wide_fused_matches_single_gpu(world):
    """The fused path at 4 and 8 ranks (rows per rank down to 8, KV heads
    replicated where there are fewer than ranks)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    cfg = _cfg(True)
    m = DecoderLM(cfg, torch.device("cuda", 0), torch.bfloat16).init_random(5, std=0.2)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=8), max_model_len=256,
                                          graph_buckets=(1, 2, 4, 8)))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 7, 33)]
    ref = eng.generate(prompts, max_tokens=12)
    fused, ok, st = _run("fused", world, wide=True)
    assert ok and all(v == 0 for v in st.values()), st
    agree = sum(a == b for x, y in zip(fused, ref) for a, b in zip(x, y)) / 36
    assert agree >= 0.75, (fused, ref)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_nvls_combine_matches_single_gpu(world):
    """B200LM_TP_NVLS=1: the partial rows stay on their rank and the combine
    reads their sum through the NVSwitch (multimem.ld_reduce on a multicast
    address); tokens agree with the single-GPU engine."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig

    cfg = _cfg(True)
    m = DecoderLM(cfg, torch.device("cuda", 0), torch.bfloat16).init_random(5, std=0.2)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=8), max_model_len=256,
                                          graph_buckets=(1, 2, 4, 8)))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 7, 33)]
    ref = eng.generate(prompts, max_tokens=12)
    fused, ok, st, on = _run("fused", world, wide=True, nvls=True)
    if not on:
        pytest.skip("no NVLink multicast on this system")
    assert ok and all(v == 0 for v in st.values()), st
    agree = sum(a == b for x, y in zip(fused, ref) for a, b in zip(x, y)) / 36
    assert agree >= 0.75, (fused, ref)
