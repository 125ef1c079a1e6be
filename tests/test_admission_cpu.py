"""Admission ledger: per-layer-kind bytes, page-granular charges, fixed and
auxiliary bytes, the watermark for new requests, and the scheduler holding
new requests back while running rows keep growing."""
from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.admission import AdmissionConfig, AdmissionLedger, LayerKind, layer_kinds_for
from mlx_swift_lm_b200.engine.types import Request, SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3

import torch


def test_bytes_and_watermark():
    kinds = [LayerKind(2, 2, 64), LayerKind(2, 2, 64, window=128), LayerKind(1, 2, 64, shared=True)]
    led = AdmissionLedger(kinds, capacity_bytes=10 * 16 * 2048, config=AdmissionConfig(
        watermark_fraction=0.1, fixed_bytes_per_request=100, auxiliary_bytes_per_token=8,
        auxiliary_token_granularity=4))
    assert led.kv_bytes_per_token == 2 * 4 * 2 * 64 * 2  # shared layers own nothing
    # 17 tokens -> two pages of KV, 20 tokens of auxiliary state
    pt = led.kv_bytes_per_token
    assert led.bytes_for(17) == 32 * pt + 20 * 8
    assert led.reserve(1, 17) and led.reserved_bytes == 32 * pt + 160 + 100
    led.reserve(1, 10)  # monotonic
    assert led.reserved_bytes == 32 * pt + 160 + 100
    led.unreserve(1, 0)
    assert led.reserved_bytes == 100
    led.release_all(1)
    assert led.reserved_bytes == 0
    cap = led.capacity_bytes
    # a new request must leave the watermark free; a running row may use it
    n = (int(cap * 0.9) - 100) // (pt + 8) // 16 * 16 - 16
    assert led.has_headroom(n, new_request=True)
    assert not led.has_headroom(n + 32, new_request=True)
    assert led.has_headroom(n + 32, new_request=False)
    assert not led.can_ever_fit(cap // pt + 16)
    s = led.snapshot()
    assert s.capacity_bytes == cap and s.watermark_bytes == int(cap * 0.1)


def test_layer_kinds_from_model():
    cfg = tiny_qwen3()
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(0)
    kinds = layer_kinds_for(m)
    assert sum(k.layers for k in kinds) == cfg.num_layers
    assert sum(k.bytes_per_token() for k in kinds) == m.kv_bytes_per_token()


def test_engine_holds_new_requests_at_the_watermark():
    cfg = tiny_qwen3()
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(1, std=0.2)
    # a ledger so small that two 100-token prompts cannot both be admitted
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=256,
                                                                    max_batched_tokens_per_step=1024),
                                          max_model_len=256, kv_tokens=1024,
                                          admission=AdmissionConfig(watermark_fraction=0.0)))
    per_tok = eng.ledger.kv_bytes_per_token
    eng.ledger.update_capacity(200 * per_tok)
    a = eng.submit(Request(prompt_tokens=list(range(100)), max_tokens=8, sampling=SamplingParams(temperature=0)))
    b = eng.submit(Request(prompt_tokens=list(range(100)), max_tokens=8, sampling=SamplingParams(temperature=0)))
    eng.step()
    assert len(eng.sched.running) == 1 and len(eng.sched.waiting) == 1
    snap = eng.capacity()
    assert snap.ledger_bytes_reserved == 112 * per_tok and snap.ledger_bytes_capacity == 200 * per_tok
    eng.run_until_idle()
    assert len(a.tokens()) == 8 and len(b.tokens()) == 8
    assert eng.ledger.reserved_bytes == 0
