"""Hybrid (Gated DeltaNet + attention) decoder on CPU: the paged engine path
with recurrent-state slots reproduces the dense single-sequence forward, and
chunked prefill carries the conv / delta-rule state exactly."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops import reference as ref


def hybrid_cfg():
    c = tiny_qwen3()
    c.model_type = "qwen3_next"
    c.layer_types = ["linear_attention", "linear_attention", "linear_attention", "full_attention"]
    c.attn_output_gate = True
    c.linear_num_key_heads, c.linear_num_value_heads = 2, 4
    c.linear_key_head_dim = c.linear_value_head_dim = 64
    return c


def test_gdn_ref_chunking_is_exact():
    torch.manual_seed(0)
    Hk, Dk, Hv, Dv = 2, 16, 4, 8
    C = 2 * Hk * Dk + Hv * Dv
    T = 11
    P = torch.randn(T, C + Hv * Dv + 2 * Hv)
    conv_w, A_log, dt_bias = torch.randn(C, 4) * 0.5, torch.rand(Hv) * 2, torch.randn(Hv)
    norm_w = torch.rand(Dv) + 0.5
    args = (conv_w, A_log, dt_bias, norm_w, Hk, Dk, Hv, Dv, 1e-6)

    def fresh_state():
        return torch.zeros(1, 3, C), torch.zeros(1, Hv, Dv, Dk)

    cs, ss = fresh_state()
    whole = ref.gdn_layer_ref(P, [0, T], [1], [0], cs, ss, *args)
    cs2, ss2 = fresh_state()
    parts = []
    for a, b in [(0, 2), (2, 3), (3, 9), (9, 11)]:  # chunks shorter than the conv window too
        parts.append(ref.gdn_layer_ref(P[a:b], [0, b - a], [1 if a == 0 else 0], [0], cs2, ss2, *args))
    assert torch.allclose(torch.cat(parts), whole, atol=1e-5)
    assert torch.allclose(ss2, ss, atol=1e-6) and torch.equal(cs2, cs)


def _eng(m, **kw):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=7),
                                           max_model_len=128, use_cuda_graphs=False, **kw))


def test_hybrid_engine_matches_dense_forward():
    m = DecoderLM(hybrid_cfg(), "cpu", torch.float32).init_random(1, std=0.2)
    assert m.num_kv_layers == 1 and [L.linear for L in m.layers] == [True, True, True, False]
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 19, 12)]
    eng = _eng(m)
    assert eng.kv.rec is not None and eng.prefix_cache is None
    out = eng.generate(prompts, max_tokens=8)
    for p, o in zip(prompts, out):
        cache = m.new_cache()
        logits = m.forward_dense(torch.tensor(p), cache)
        want = []
        for _ in range(8):
            t = int(logits[-1].argmax())
            want.append(t)
            logits = m.forward_dense(torch.tensor([t]), cache)
        assert o == want
    assert eng.kv.rec.num_free == 4  # every slot returned


def test_hybrid_checkpoint_roundtrip(tmp_path):
    from mlx_swift_lm_b200.loader.convert import save_model
    from mlx_swift_lm_b200.loader.load import load_model

    m = DecoderLM(hybrid_cfg(), "cpu", torch.float32).init_random(4, std=0.2)
    d = str(tmp_path / "hyb")
    save_model(m, d, dtype=torch.float32)
    m2, hf = load_model(d, device="cpu", dtype=torch.float32)
    assert hf["model_type"] == "qwen3_next" and m2.cfg.layer_types == m.cfg.layer_types
    toks = torch.arange(3, 30)
    a = m2.forward_dense(toks, m2.new_cache())
    b = m.forward_dense(toks, m.new_cache())
    assert torch.allclose(a, b, atol=1e-4)
