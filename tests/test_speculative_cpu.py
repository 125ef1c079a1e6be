"""Single-request speculative decoding: a draft-model iterator and the MTP
engine path both reproduce plain greedy decoding."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.api.generate import GenerateParameters, SpeculativeTokenIterator, TokenIterator, generate_mtp
from mlx_swift_lm_b200.models.config import tiny_qwen3


def test_draft_model_iterator_matches_greedy():
    target = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(1, std=0.2)
    cfg = tiny_qwen3()
    cfg.num_layers = 2
    draft = DecoderLM(cfg, "cpu", torch.float32).init_random(1, std=0.2)  # shares the first layers' seed stream
    prompt = list(range(3, 20))
    p = GenerateParameters(temperature=0.0, max_tokens=24)
    want = list(TokenIterator(target, prompt, p))
    for k in (1, 2, 4):
        it = SpeculativeTokenIterator(target, draft, prompt, p, num_draft=k)
        assert list(it) == want, k
        assert 0.0 <= it.acceptance_rate <= 1.0
        assert it.dcache.offset == it.cache.offset  # the draft stays in step with the target
    self_spec = SpeculativeTokenIterator(target, target, prompt, p, num_draft=3)
    assert list(self_spec) == want and self_spec.acceptance_rate == 1.0


def test_generate_mtp_single_request():
    from mlx_swift_lm_b200.engine.mtp import MTPConfig
    from mlx_swift_lm_b200.models.mtp import MTPModule

    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(2, std=0.2)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=128,
                                          use_cuda_graphs=False))
    plain, _, _ = __import__("mlx_swift_lm_b200.api.generate", fromlist=["generate"]).generate(
        eng, list(range(5, 30)), GenerateParameters(temperature=0.0, max_tokens=16))
    eng.enable_mtp(MTPModule(m).init_random(3, std=0.2), MTPConfig(k=2))
    toks, _, _, tele = generate_mtp(eng, list(range(5, 30)), GenerateParameters(temperature=0.0, max_tokens=16))
    assert toks == plain and tele["rounds"] > 0 and tele["drafted"] == 2 * tele["rounds"]
