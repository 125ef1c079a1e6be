"""Engine diagnostics: step profiler records, attention-metadata capture and
replay reproduce the step's logits, logit reports, teacher-forced scores."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.engine.diagnostics import Diagnostics, replay_batch, teacher_forced_scores
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _eng():
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(5, std=0.2)
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=128,
                                           use_cuda_graphs=False))


def test_profile_capture_and_logits():
    eng = _eng()
    eng.diagnostics = Diagnostics(profile=True, capture_attention=True, logit_topk=3)
    eng.submit(Request(prompt_tokens=list(range(1, 20)), max_tokens=4))
    eng.submit(Request(prompt_tokens=list(range(5, 9)), max_tokens=4))
    eng.run_until_idle()
    s = eng.diagnostics.step_summary()
    assert s["forwards"] >= 4 and s["wall_ms"]["p50"] > 0 and s["tokens"] > 0
    rep = eng.diagnostics.logits[0]
    assert len(rep.top_ids) == 3 and rep.non_finite == 0 and rep.entropy > 0
    # replaying a captured decode step on the same KV state reproduces its logits
    eng2 = _eng()
    eng2.diagnostics = Diagnostics(capture_attention=True)
    eng2.submit(Request(prompt_tokens=list(range(1, 20)), max_tokens=3))
    eng2.step()
    eng2.step()
    meta = eng2.diagnostics.captures[-1]
    fb = replay_batch(meta, eng2.device)
    a = eng2.model.forward(fb, eng2.kv)
    b = eng2.model.forward(replay_batch(meta, eng2.device), eng2.kv)
    assert torch.equal(a, b)


def test_teacher_forced_scores():
    eng = _eng()
    prompt, cont = [3, 4, 5, 6], [7, 8, 9]
    sc = teacher_forced_scores(eng, prompt, cont)
    m = eng.model
    lg = m.forward_dense(torch.tensor(prompt + cont), m.new_cache())
    lp = torch.log_softmax(lg.float(), -1)
    want = [lp[len(prompt) - 1 + i, t].item() for i, t in enumerate(cont)]
    assert all(abs(x - y) < 1e-4 for x, y in zip(sc, want))
