"""Engine safety: the step watchdog ends every live stream when a step wedges
(a scripted host-side sleep inside the forward), and a churn storm of
submits / cancels / finishes leaves every surviving request's tokens equal to
the same request run alone (batch-composition invariance)."""
import random
import threading
import time

import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.types import FinishReason, Request, SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.testing.scripted import ScriptedLM

EOS = 302


def test_watchdog_finishes_every_stream_on_a_wedged_step():
    release = threading.Event()

    class Wedge(ScriptedLM):
        calls = 0

        def forward(self, fb, kv, **kw):
            Wedge.calls += 1
            if Wedge.calls == 3:  # the third step never returns in time
                release.wait(10.0)
            return super().forward(fb, kv, **kw)

    m = Wedge([10, 11, 12, 13, 14, 15, 16, 17, 18, EOS], prompt_len=4)
    wedged = []
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4), max_model_len=64,
                                          step_timeout_s=0.3), eos_token_ids=[EOS])
    eng.on_step_wedge = lambda: wedged.append(True)
    streams = [eng.submit(Request(prompt_tokens=[1, 2, 3, 4], max_tokens=9, sampling=SamplingParams(temperature=0.0)))
               for _ in range(3)]
    eng.start()
    try:
        finals = []
        for s in streams:
            t_end = time.time() + 5.0
            fin = None
            while time.time() < t_end:
                ev = s.get(timeout=0.1)
                if ev is not None and ev.finished:
                    fin = ev
                    break
            finals.append(fin)
        assert all(f is not None for f in finals), "a stream never finished"
        assert all(f.finish_reason == FinishReason.WATCHDOG and f.cause == "watchdog" for f in finals)
        assert wedged == [True] and not eng.healthy
    finally:
        release.set()
        eng.shutdown(timeout=5.0)


def _solo(model, req_kw):
    eng = EngineV2(model, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=1), max_model_len=256))
    s = eng.submit(Request(**req_kw))
    eng.run_until_idle()
    return s.tokens()


def test_churn_storm_invariance():
    torch.manual_seed(0)
    cfg = tiny_qwen3()
    model = DecoderLM(cfg, "cpu", torch.float32).init_random(9, std=0.3)
    rng = random.Random(5)
    eng = EngineV2(model, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=6,
                                                                        max_batched_tokens_per_step=96,
                                                                        prefill_chunk_size=32),
                                              max_model_len=256))
    live, kws, cancelled = {}, {}, set()
    for step in range(60):
        if step < 40 and rng.random() < 0.4:
            kw = dict(prompt_tokens=[rng.randrange(cfg.vocab_size) for _ in range(rng.randint(3, 70))],
                      max_tokens=rng.randint(2, 14), sampling=SamplingParams(temperature=0.0))
            s = eng.submit(Request(**kw))
            live[s.request_id] = s
            kws[s.request_id] = kw
        if live and rng.random() < 0.08:
            rid = rng.choice(sorted(live))
            if eng.cancel(rid):
                cancelled.add(rid)
        eng.step()
    eng.run_until_idle()
    done = [rid for rid in live if rid not in cancelled]
    assert len(done) >= 8
    for rid in done:
        assert live[rid].tokens() == _solo(model, kws[rid]), rid
