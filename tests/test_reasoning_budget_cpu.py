"""Reasoning budget: the thought is cut at the budget by forcing the closer,
the opener is banned once a thought opened or closed, the state follows
confirmed tokens only, and rule violations end the request with an error."""
import pytest

from mlx_swift_lm_b200 import EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.reasoning import ReasoningBudget, ReasoningBudgetState
from mlx_swift_lm_b200.engine.types import FinishReason, Request, SamplingParams
from mlx_swift_lm_b200.testing.scripted import ScriptedLM

OPEN, CLOSE, EOS = 300, 301, 302


def _run(script, budget, prompt_len=5, markers=(OPEN, CLOSE), max_tokens=12):
    m = ScriptedLM(script, prompt_len=prompt_len)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=128,
                                          reasoning_markers=markers), eos_token_ids=[EOS])
    s = eng.submit(Request(prompt_tokens=list(range(1, prompt_len + 1)), max_tokens=max_tokens,
                           sampling=SamplingParams(temperature=0.0), reasoning_budget=budget))
    eng.run_until_idle()
    return s.tokens(), s.st


def test_budget_forces_closer_and_bans_second_opener():
    script = [OPEN, 10, 11, 12, 13, 14, CLOSE, 20, OPEN, 21, EOS]
    out, st = _run(script, budget=2)
    # two thought tokens, then the closer is forced in place of 12
    assert out[:4] == [OPEN, 10, 11, CLOSE]
    assert OPEN not in out[1:]
    assert st.extra["budget"].consumed == 2


def test_budget_not_reached_leaves_output_unchanged():
    script = [OPEN, 10, CLOSE, 20, 21, EOS]
    out, _ = _run(script, budget=5)
    assert out == [OPEN, 10, CLOSE, 20, 21, EOS]


def test_budget_starting_inside_thought():
    script = [10, 11, 12, CLOSE, 20, EOS]
    out, _ = _run(script, budget=1, markers=(OPEN, CLOSE, True))
    assert out[:2] == [10, CLOSE]


def test_budget_needs_markers_and_valid_config():
    with pytest.raises(ValueError, match="marker"):
        _run([10, EOS], budget=3, markers=None)
    with pytest.raises(ValueError):
        ReasoningBudget(0, OPEN, CLOSE)
    with pytest.raises(ValueError):
        ReasoningBudget(4, OPEN, OPEN)


def test_budget_state_records_violations():
    st = ReasoningBudgetState(ReasoningBudget(1, OPEN, CLOSE), history=[OPEN, 7])
    assert st.forced() == CLOSE
    st.confirm(8)  # a thought token past the limit (a path that ignored the forced closer)
    assert st.failure is not None
    st2 = ReasoningBudgetState(ReasoningBudget(3, OPEN, CLOSE), history=[OPEN, CLOSE, OPEN])
    assert "opener" in st2.failure


def test_budget_violation_ends_request_with_error():
    m = ScriptedLM([OPEN, 10, 11, EOS], prompt_len=5)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=64,
                                          reasoning_markers=(OPEN, CLOSE)), eos_token_ids=[EOS])
    s = eng.submit(Request(prompt_tokens=[1, 2, 3, 4, 5], max_tokens=8, sampling=SamplingParams(temperature=0.0),
                           reasoning_budget=1))
    # a confirmed stream that already broke the rule (e.g. replayed history)
    s.st.extra["budget"].failure = "reasoning budget: token beyond thought limit"
    eng.run_until_idle()
    evs = []
    while True:
        ev = s.get(timeout=0)
        if ev is None:
            break
        evs.append(ev)
    fin = [e for e in evs if e.finished]
    assert fin and fin[-1].finish_reason == FinishReason.ERROR


def test_non_finite_logits_end_the_row_with_an_error():
    """A row whose logits hold NaN ends with an error and commits nothing from
    that position; its batch-mate is unaffected."""
    from mlx_swift_lm_b200.engine.engine import NON_FINITE_MESSAGE

    class NaNAt(ScriptedLM):
        def forward(self, fb, kv, **kw):
            lg = super().forward(fb, kv, **kw)
            pos = fb.positions if fb.logit_idx is None else fb.positions[fb.logit_idx]
            lg[(pos == 7).nonzero().flatten()] = float("nan")
            return lg

    m = NaNAt([10, 11, 12, 13, 14, 15, EOS], prompt_len=5)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=64),
                   eos_token_ids=[EOS])
    bad = eng.submit(Request(prompt_tokens=[1, 2, 3, 4, 5], max_tokens=8, sampling=SamplingParams(temperature=0.0)))
    good = eng.submit(Request(prompt_tokens=[1, 2, 3, 4, 5, 6, 7, 8, 9], max_tokens=3,
                              sampling=SamplingParams(temperature=0.0)))
    eng.run_until_idle()
    evs = []
    while (ev := bad.get(timeout=0)) is not None:
        evs.append(ev)
    fin = evs[-1]
    assert fin.finished and fin.finish_reason == FinishReason.ERROR and fin.error == NON_FINITE_MESSAGE
    # the logits at positions 4, 5, 6 produced tokens; position 7's NaN row committed nothing
    assert [t for e in evs for t in e.tokens] == [10, 11, 12]
    assert len(good.tokens()) == 3 and eng.non_finite_rows == 1
