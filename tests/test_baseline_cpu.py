"""The stock-PyTorch comparison build computes the same function as the
framework's decoder: same seeded weights, same engine, same greedy tokens
(tiny Qwen3 on CPU in fp32), and it refuses model features it does not
implement."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.baseline import TorchDecoderLM
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _engine(model, prefill_chunk=4096):
    eng = EngineV2(model, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4,
                                                                        prefill_chunk_size=prefill_chunk),
                                              max_model_len=256))
    if isinstance(model, TorchDecoderLM):
        model.bind_engine(eng)
    return eng


@pytest.mark.parametrize("chunk", [4096, 16])
def test_baseline_matches_framework_model(chunk):
    cfg = tiny_qwen3()
    ours = DecoderLM(cfg, "cpu", torch.float32).init_random(3, std=0.2)
    base = TorchDecoderLM(cfg, "cpu", torch.float32).init_random(3, std=0.2)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (33, 5, 70)]
    want = _engine(ours).generate(prompts, max_tokens=12)
    got = _engine(base, prefill_chunk=chunk).generate(prompts, max_tokens=12)
    assert got == want


def test_baseline_logits_close():
    cfg = tiny_qwen3()
    ours = DecoderLM(cfg, "cpu", torch.float32).init_random(5, std=0.2)
    base = TorchDecoderLM(cfg, "cpu", torch.float32).init_random(5, std=0.2)
    from mlx_swift_lm_b200.kv.paged import PagedKVCache
    from mlx_swift_lm_b200.models.batch import ForwardBatch

    toks = torch.arange(40) % cfg.vocab_size
    outs = []
    for m in (ours, base):
        kv = PagedKVCache.for_model(m, max_tokens=256)
        pages = kv.pool.alloc(4)
        if isinstance(m, TorchDecoderLM):
            m.scratch_page = kv.pool.alloc(1)[0]
        slots = torch.tensor([pages[i // 16] * 16 + i % 16 for i in range(40)], dtype=torch.int64)
        fb = ForwardBatch(input_ids=toks.to(torch.int32), positions=torch.arange(40, dtype=torch.int32), slots=slots,
                          pf_cu_q=torch.tensor([0, 40], dtype=torch.int32), pf_cu_q_host=[0, 40],
                          pf_pos0=torch.zeros(1, dtype=torch.int32), pf_pos0_host=[0],
                          pf_page_table=torch.tensor([pages], dtype=torch.int32))
        outs.append(m.forward(fb, kv))
    torch.testing.assert_close(outs[1], outs[0], atol=2e-4, rtol=2e-4)


def test_baseline_refuses_unsupported_features():
    cfg = tiny_qwen3()
    cfg.attention_sinks = True
    m = TorchDecoderLM(cfg, "cpu", torch.float32).init_random(1)
    with pytest.raises(ValueError, match="sinks"):
        m.check_supported()
