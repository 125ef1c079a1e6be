"""Prefix caching for hybrid models (Gated DeltaNet + attention) on CPU: the
recurrent state is kept at the prompt's last full block boundary, a later
request with the same prefix adopts the blocks' KV pages plus the state
snapshot and computes only the rest, and its tokens equal an uncached run."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.engine.types import SamplingParams

from test_gdn_cpu import hybrid_cfg


def _eng(m, cache=True, snaps=4):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=48),
                                           max_model_len=256, use_cuda_graphs=False, enable_prefix_cache=cache,
                                           prefix_block_size=32, prefix_state_snapshots=snaps))


def _run(eng, prompt, n=8):
    s = eng.submit(Request(prompt_tokens=prompt, max_tokens=n, sampling=SamplingParams(temperature=0.0)))
    eng.run_until_idle()
    return s.tokens(), s


def test_hybrid_prefix_reuse_matches_uncached():
    m = DecoderLM(hybrid_cfg(), "cpu", torch.float32).init_random(3, std=0.1)
    g = torch.Generator().manual_seed(5)
    shared = torch.randint(0, m.cfg.vocab_size, (100,), generator=g).tolist()
    a = shared + torch.randint(0, m.cfg.vocab_size, (9,), generator=g).tolist()
    b = shared + torch.randint(0, m.cfg.vocab_size, (13,), generator=g).tolist()
    ref_b, _ = _run(_eng(m, cache=False), b)
    eng = _eng(m)
    pc = eng.prefix_cache
    assert pc is not None and pc.states is not None
    _run(eng, a)
    assert pc.states.saves >= 1  # state kept at block 96 (the last full block before a's last token)
    out_b, sb = _run(eng, b)
    assert out_b == ref_b
    assert pc.states.restores == 1 and sb.st.usage.cached_prompt_tokens == 96
    # no snapshot slots: hybrid models run without a prefix cache
    assert _eng(m, snaps=0).prefix_cache is None


def test_hybrid_prefix_chunk_stops_at_boundary():
    m = DecoderLM(hybrid_cfg(), "cpu", torch.float32).init_random(4, std=0.1)
    eng = _eng(m)
    p = list(range(1, 71))  # boundary at 64: chunks 48 then 16 (stop at 64), then 6
    s = eng.submit(Request(prompt_tokens=p, max_tokens=2, sampling=SamplingParams(temperature=0.0)))
    chunks = []
    while s.st.status.name != "FINISHED":
        eng.step()
        chunks.append(s.st.num_computed)
    assert 64 in chunks  # one chunk ended exactly at the snapshot boundary
    assert eng.prefix_cache.states.saves >= 1
