"""Data-parallel serving: engine replicas behind one router compute exactly
what one engine computes, spread load, keep prefix affinity, cancel through
the owner, and aggregate capacity."""
import torch

from mlx_swift_lm_b200 import EngineConfig, SchedulerConfig
from mlx_swift_lm_b200.api.container import ModelContainer
from mlx_swift_lm_b200.engine.types import Request, SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _container():
    ecfg = EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4), max_model_len=512,
                        use_cuda_graphs=False)
    return ModelContainer.random(tiny_qwen3(), "cpu", torch.float32, seed=3, std=0.2, engine_config=ecfg)


def test_replicas_route_and_match_single_engine():
    single = _container()
    dp = _container().replicate(["cpu"])
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (30, 300, 12, 260, 7, 90)]
    want = single.engine.generate(prompts, max_tokens=8)
    streams = [dp.engine.submit(Request(prompt_tokens=p, max_tokens=8, sampling=SamplingParams(temperature=0)))
               for p in prompts]
    dp.engine.run_until_idle()
    assert [s.tokens() for s in streams] == want
    assert min(dp.engine.routed) >= 2  # both replicas served
    cap = dp.engine.capacity()
    assert cap.kv_pages_total == 2 * single.engine.capacity().kv_pages_total


def test_prefix_affinity_and_cancel():
    dp = _container().replicate(["cpu"])
    base = list(range(1, 257))
    a = Request(prompt_tokens=base + [5], max_tokens=4)
    b = Request(prompt_tokens=base + [6, 7], max_tokens=4)
    ia = dp.engine.route(a)
    ib = dp.engine.route(b)
    assert ia == ib  # same first block -> same replica
    r = dp.engine.submit(Request(prompt_tokens=[1, 2, 3], max_tokens=50))
    assert dp.engine.cancel(r.request_id)
