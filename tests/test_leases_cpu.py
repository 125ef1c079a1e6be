"""Deadline leases and first-token deadline admission with an injected clock
(no sleeps): typed causes, progress refresh, backpressure, safety ceiling."""
import math

import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.engine.leases import (FirstTokenDeadline, LeaseConfig, RequestLeases, TerminalCause,
                                             safety_ceiling_s)
from mlx_swift_lm_b200.models.config import tiny_qwen3


def test_lease_state_machine():
    cfg = LeaseConfig(admission_s=10, prefill_s=5, decode_s=3, backpressure_s=7, decode_floor_tps=1.0)
    ls = RequestLeases(0.0, cfg, prompt_tokens=400, max_tokens=100)
    assert ls.expired_cause(9.0, False) is None
    assert ls.expired_cause(10.5, False) == TerminalCause.ADMISSION_TIMEOUT
    ls.mark_admitted(10.0)
    assert ls.expired_cause(14.0, True) is None
    assert ls.expired_cause(15.5, True) == TerminalCause.PREFILL_STALL
    ls.record_progress(15.0, computed=100, generated=0)  # prefill progress refreshes
    assert ls.expired_cause(19.0, True) is None
    ls.record_progress(19.0, computed=400, generated=1)  # first token: decode lease
    assert ls.expired_cause(22.5, True) == TerminalCause.DECODE_STALL
    for t in range(20, 60):  # a request that keeps producing tokens never stalls
        ls.record_progress(float(t), 400, t)
        assert ls.expired_cause(t + 2.0, True) is None
    ls.mark_paused(60.0)
    assert ls.expired_cause(66.0, True) is None
    assert ls.expired_cause(67.5, True) == TerminalCause.BACKPRESSURE_TIMEOUT
    ls.mark_resumed(67.0)
    ceiling = safety_ceiling_s(400, 100, cfg)
    assert ceiling == 10 + 2 * 400 / 200 + 100 / 1.0 + 60
    assert ls.expired_cause(ceiling + 0.1, True) == TerminalCause.SAFETY_DEADLINE


class FakeClock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t


def test_engine_admission_lease_and_first_token_deadline():
    clock = FakeClock()
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(1)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=1), max_model_len=128,
                                          use_cuda_graphs=False, clock=clock,
                                          leases=LeaseConfig(admission_s=5, decode_floor_tps=0)))
    a = eng.submit(Request(prompt_tokens=list(range(1, 30)), max_tokens=50))
    b = eng.submit(Request(prompt_tokens=list(range(1, 10)), max_tokens=5))  # waits: one slot
    eng.step()
    clock.t = 6.0
    eng.step()
    ev = [e for e in b.q if e.finished]
    assert ev and ev[0].cause == TerminalCause.ADMISSION_TIMEOUT
    # first-token deadline: no decode rate while rows decode -> fail closed
    r = eng.submit(Request(prompt_tokens=[1, 2, 3], max_tokens=2,
                           first_token_deadline=FirstTokenDeadline(deadline=clock.t + 100.0, prefill_tps=1000.0)))
    assert r.q[0].cause == TerminalCause.FIRST_TOKEN_DEADLINE
    ok = eng.submit(Request(prompt_tokens=[1, 2, 3], max_tokens=2,
                            first_token_deadline=FirstTokenDeadline(deadline=clock.t + 100.0, prefill_tps=1000.0,
                                                                    decode_tps=1000.0)))
    assert not ok.q
    eng.run_until_idle()
    assert a.st.num_output == 50
