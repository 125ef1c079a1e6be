"""Adaptive MTP depth: the controller moves toward the depth with the most
expected tokens per unit of round time, probes neighbours, and the engine's
MTP rounds run under it with bounded drafter rows."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.mtp import MTPConfig
from mlx_swift_lm_b200.engine.mtp_depth import DepthController
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.models.mtp import MTPModule


def _simulate(acc_rate, cost_per_draft, rounds=400, k_max=6, seed=0):
    import random

    rng = random.Random(seed)
    c = DepthController(k_max)
    for _ in range(rounds):
        k = c.choose()
        acc = []
        for _row in range(8):
            a = 0
            while a < k and rng.random() < acc_rate:
                a += 1
            acc.append(a)
        c.observe(k, acc, 1.0 + cost_per_draft * k)
    return c


def test_high_acceptance_cheap_drafts_goes_deep():
    c = _simulate(0.9, 0.05)
    assert c.depth >= 4


def test_low_acceptance_expensive_drafts_stays_shallow():
    c = _simulate(0.2, 0.5)
    assert c.depth <= 2


def test_expected_tokens_formula():
    c = DepthController(3)
    for _ in range(20):
        c.observe(3, [3], 1.0)  # every draft accepted
    assert abs(c.expected_tokens(3) - 4.0) < 1e-6
    c2 = DepthController(2)
    for _ in range(200):
        c2.observe(2, [0], 1.0)  # first draft always rejected
    assert c2.rate(1) < 0.01 and c2.expected_tokens(2) < 1.02


def test_engine_adaptive_mtp_and_row_cap():
    cfg = tiny_qwen3()
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(2, std=0.2)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4), max_model_len=256))
    drv = eng.enable_mtp(MTPModule(m).init_random(3, std=0.2),
                         MTPConfig(k=3, acceptance="bernoulli", p=0.8, adaptive=True, max_rows=2))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 20)]
    out = eng.generate(prompts, max_tokens=40)
    assert all(len(o) == 40 for o in out)
    assert drv.stats.rounds > 0 and drv.depth.rounds == drv.stats.rounds
    # three decode rows exceed max_rows: those steps decode without drafts
    eng2 = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4), max_model_len=256))
    drv2 = eng2.enable_mtp(MTPModule(m).init_random(3, std=0.2), MTPConfig(k=2, max_rows=2))
    out2 = eng2.generate(prompts + [prompts[0]], max_tokens=10)
    assert all(len(o) == 10 for o in out2) and drv2.stats.rounds == 0
