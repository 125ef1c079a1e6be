"""Multi-process tests on CPU (gloo, world size 2): tensor-parallel sharding
computes the same function as one rank; collectives and failure handling on
the host."""
import os
import queue
import time
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


def _guard_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
    from mlx_swift_lm_b200.engine.types import Request
    from mlx_swift_lm_b200.models.config import tiny_qwen3
    from mlx_swift_lm_b200.models.decoder import TensorParallel
    from mlx_swift_lm_b200.parallel.health import CommGuard

    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32, tp=TensorParallel(rank, world, dist.group.WORLD)).init_random(
        3, std=0.2)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=64,
                                          use_cuda_graphs=False))
    aborted = []
    CommGuard(eng, dist.group.WORLD, abort_fn=lambda g: aborted.append(True))
    s = eng.submit(Request(prompt_tokens=[5, 6, 7, 8], max_tokens=20))
    for _ in range(3):  # both ranks step together
        eng.step()
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    for _ in range(30):
        if not eng.healthy:
            break
        eng.step()
    evs = list(s.q)
    q.put((eng.healthy, bool(aborted), evs[-1].cause if evs else None, evs[-1].finished if evs else None))


def test_comm_guard_aborts_on_dead_rank():
    """A rank that leaves: the survivor's next collective times out, the guard
    aborts the communicator, the engine turns unhealthy and the stream ends
    with cause comm_abort (no hang)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_guard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res, t0 = None, time.monotonic()
    while res is None and time.monotonic() - t0 < 180:
        try:
            res = q.get(timeout=2)
        except queue.Empty:
            if ps[0].exitcode not in (None, 0):  # the survivor raised instead of reporting
                break
    assert res is not None, f"survivor exit code {ps[0].exitcode}"
    healthy, aborted, cause, finished = res
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert not healthy and aborted and cause == "comm_abort" and finished


def test_comm_guard_reads_kernel_status():
    class Eng:
        healthy = True
        on_step_wedge = None
        states = {}

    from mlx_swift_lm_b200.parallel.health import CommGuard

    calls = []
    e = Eng()
    g = CommGuard(e, None, abort_fn=lambda grp: calls.append(grp), check_every=2,
                  read_status=lambda clear=False: {"gemm": 0, "tp": 4})
    g.after_step(1)
    assert e.healthy
    g.after_step(2)
    assert not e.healthy and calls == [None] and "collective wait expired" in g.aborted
    e2 = Eng()
    g2 = CommGuard(e2, None, abort_fn=lambda grp: calls.append("w"))
    e2.on_step_wedge()  # the watchdog's wedge callback aborts too
    assert not e2.healthy and calls[-1] == "w"


def test_nvls_buffer_falls_back_without_multicast():
    """Where the system offers no NVLink multicast (here: a CPU gloo group),
    the NVLS buffer request warns and returns None, so the fused TP keeps the
    push-to-every-rank exchange."""
    from mlx_swift_lm_b200.parallel.tp_fused import nvls_buffer

    if dist.is_initialized():
        pytest.skip("a default process group already exists in this process")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1)
    try:
        with pytest.warns(UserWarning, match="NVLS"):
            assert nvls_buffer(dist.group.WORLD, (2, 8, 16), torch.device("cpu")) is None
    finally:
        dist.destroy_process_group()
