"""Sliding-window ring storage: windowed layers keep window + one step of
pages per sequence (page p on ring page p % R) in a pool of their own, full
layers keep growing pages. Generation through the paged engine is identical
with and without rings (greedy, chunked prefill crossing the window, decode
past several wraps), and a sequence never holds more than R ring pages."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.kv.paged import ring_pages_for
from mlx_swift_lm_b200.models.families import build_config


def _cfg(mt="gemma3_text", **kw):
    d = dict(model_type=mt, vocab_size=300, hidden_size=64, num_hidden_layers=4, num_attention_heads=2,
             num_key_value_heads=1, head_dim=32, intermediate_size=128, rms_norm_eps=1e-6, rope_theta=10000.0,
             max_position_embeddings=2048, sliding_window=24, sliding_window_pattern=2, query_pre_attn_scalar=32,
             rope_local_base_freq=10000.0)
    d.update(kw)
    return build_config(d)


def _engine(m, ring, chunk=10):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=3, prefill_chunk_size=chunk),
                                           max_model_len=256, use_cuda_graphs=False, window_ring=ring))


def test_ring_matches_full_storage():
    cfg = _cfg()
    assert cfg.layer_windows == [24, 0, 24, 0]
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(0, std=0.2)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 300, (n,), generator=g).tolist() for n in (5, 61, 33)]
    ref = _engine(m, False).generate(prompts, max_tokens=40)
    e = _engine(m, True)
    assert e.kv.ring_pages == ring_pages_for(24, 11)
    assert e.kv.layer_ring == [True, False, True, False]
    assert e.kv.gk[0].shape[1] == 3 * e.kv.ring_pages + 1  # ring pool: max_concurrent rings
    got = e.generate(prompts, max_tokens=40)
    assert got == ref


def test_ring_holds_bounded_pages_and_releases():
    cfg = _cfg()
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(1, std=0.2)
    e = _engine(m, True)
    R = e.kv.ring_pages
    free0 = e.kv.ring_pool.num_free
    from mlx_swift_lm_b200.engine.types import Request

    e.submit(Request(prompt_tokens=list(range(1, 90)), max_tokens=60))
    peak = 0
    while e.sched.has_work() or e._inflight is not None:
        e.step()
        for st in e.sched.running:
            peak = max(peak, len(st.seq.ring))
            assert len(st.seq.ring) <= R
    e._drain_inflight()
    assert peak == R  # 149 tokens need far more than R pages of full storage
    assert e.kv.ring_pool.num_free == free0


def test_gemma4_ring_matches_full_storage():
    """Gemma 4: rings for the sliding layers, growing pages for the global
    layers (different head dims in separate slabs), KV-shared layers reading
    either kind."""
    hf = dict(model_type="gemma4_text", vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=6,
              num_attention_heads=2, num_key_value_heads=1, head_dim=32, global_head_dim=64, sliding_window=16,
              layer_types=["sliding_attention", "sliding_attention", "full_attention", "sliding_attention",
                           "sliding_attention", "full_attention"], num_kv_shared_layers=2,
              hidden_size_per_layer_input=16, vocab_size_per_layer_input=300, use_double_wide_mlp=True,
              final_logit_softcapping=30.0, max_position_embeddings=1024,
              rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
                               "full_attention": {"rope_type": "proportional", "partial_rotary_factor": 0.25,
                                                  "rope_theta": 1000000.0}})
    m = DecoderLM(build_config(hf), "cpu", torch.float32).init_random(2, std=0.15)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 300, (n,), generator=g).tolist() for n in (40, 9)]
    ref = _engine(m, False, chunk=8).generate(prompts, max_tokens=30)
    e = _engine(m, True, chunk=8)
    assert e.kv.layer_ring == [True, True, False, True]
    assert e.generate(prompts, max_tokens=30) == ref
