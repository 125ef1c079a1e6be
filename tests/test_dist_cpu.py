"""Multi-process tests on CPU (gloo, world size 2): tensor-parallel sharding
computes the same function as one rank; collectives and failure handling on
the host."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.dist


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q, seed):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from mlx_swift_lm_b200 import DecoderLM
        from mlx_swift_lm_b200.models.config import tiny_qwen3
        from mlx_swift_lm_b200.models.decoder import TensorParallel

        torch.manual_seed(0)
        cfg = tiny_qwen3()
        m = DecoderLM(cfg, "cpu", torch.float32, tp=TensorParallel(rank, world, dist.group.WORLD)).init_random(
            seed, std=0.2)
        toks = torch.arange(3, 40) % cfg.vocab_size
        lg = m.forward_dense(toks, m.new_cache())
        if rank == 0:
            # numpy pickles by value: a torch tensor would travel as a shared-memory fd
            # that the receiver can only open while this process is still alive
            q.put(lg.detach().numpy().copy())
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_matches_single_rank():
    from mlx_swift_lm_b200 import DecoderLM
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    seed = 11
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(seed, std=0.2)
    ref = m.forward_dense(torch.arange(3, 40) % 4096, m.new_cache())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_tp_worker, args=(r, 2, port, q, seed)) for r in range(2)]
    for p in ps:
        p.start()
    out = torch.from_numpy(q.get(timeout=120))
    for p in ps:
        p.join(60)
    assert all(p.exitcode == 0 for p in ps)
    assert torch.allclose(out, ref, atol=2e-4, rtol=1e-4), (out - ref).abs().max()


def _dead_rank_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # a rank that leaves between steps, before the next collective
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put("no-error")
    except Exception as e:  # the survivor learns of the failure from the collective timeout
        q.put(type(e).__name__)


def test_collective_timeout_reports_dead_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = q.get(timeout=120)
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert res != "no-error"


def _max_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    from mlx_swift_lm_b200.parallel.timing import max_over_ranks

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        out = max_over_ranks([1.0 + rank, 5.0 - rank], "cpu")
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_max_over_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_max_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = q.get(timeout=120)
    for p in ps:
        p.join(60)
    assert out == [2.0, 5.0]
