"""OLMo 2 / OLMo 3 / EXAONE 4 (post-sublayer norms only, whole-projection or
per-head q/k norms, NoPE global layers, local RoPE bases) and Gemma 3 local
RoPE: config translation, the paged engine == the dense path, and the block
math against a plain torch restatement."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.families import build_config


def _hf(mt, **kw):
    base = dict(model_type=mt, vocab_size=512, hidden_size=128, num_hidden_layers=4, num_attention_heads=4,
                num_key_value_heads=2, head_dim=32, intermediate_size=256, rms_norm_eps=1e-6, rope_theta=10000.0,
                max_position_embeddings=2048)
    base.update(kw)
    return base


def _engine_vs_dense(cfg, seed=0):
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(seed, std=0.2)
    toks = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(1))
    dense = m.forward_dense(toks, m.new_cache()).argmax(-1)[-1].item()
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2, prefill_chunk_size=16),
                                          max_model_len=256))
    out = eng.generate([toks.tolist()], max_tokens=6)[0]
    assert out[0] == dense
    ref = []
    cache = m.new_cache()
    lg = m.forward_dense(toks, cache)
    t = lg.argmax(-1)[-1]
    for _ in range(6):
        ref.append(int(t))
        t = m.forward_dense(t.view(1), cache).argmax(-1)[-1]
    assert out == ref
    return m


def test_olmo2_config_and_engine():
    cfg = build_config(_hf("olmo2"))
    assert not cfg.pre_norms and cfg.post_norms and cfg.qk_norm_full
    m = _engine_vs_dense(cfg)
    L = m.layers[0]
    assert L.ln1 is None and L.q_norm.shape[0] == 4 * 32 and L.k_norm.shape[0] == 2 * 32


def test_exaone4_pattern_nope_and_windows():
    cfg = build_config(_hf("exaone4", sliding_window=8, sliding_window_pattern="LLLG"))
    assert cfg.layer_windows == [8, 8, 8, 0] and cfg.nope_layers == [3] and cfg.qk_norm
    m = _engine_vs_dense(cfg)
    cs, rd = m.rope_for(3)
    assert rd == 0 and m.rope_for(0)[1] == 32


def test_olmo3_local_rope_base():
    cfg = build_config(_hf("olmo3", sliding_window=8, layer_types=["sliding_attention", "sliding_attention",
                                                                    "sliding_attention", "full_attention"],
                           rope_scaling={"rope_type": "yarn", "factor": 4.0,
                                         "original_max_position_embeddings": 512}))
    m = _engine_vs_dense(cfg)
    assert m.cos_sin_local is not None and not torch.equal(m.rope_for(0)[0], m.rope_for(3)[0])


def test_gemma3_local_layers_use_the_local_base():
    cfg = build_config(_hf("gemma3_text", sliding_window=8, sliding_window_pattern=2, rope_theta=1e6,
                           rope_local_base_freq=10000.0, query_pre_attn_scalar=32))
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(0)
    assert cfg.window(0) == 8 and cfg.window(1) == 0
    local, _ = m.rope_for(0)
    glob, _ = m.rope_for(1)
    # position 5, first frequency: cos(5 * base^0) is the same; the slowest frequency differs by base
    assert not torch.allclose(local[100], glob[100])


def test_post_norm_block_math():
    """One OLMo 2 layer against a plain torch restatement:
    h = x + norm(attn(x)); out = h + norm(mlp(h))."""
    cfg = build_config(_hf("olmo2", num_hidden_layers=1))
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(3, std=0.2)
    toks = torch.tensor([5, 9, 11, 3])
    got = m.forward_dense(toks, m.new_cache(), return_hidden=True)
    L = m.layers[0]
    x = m.embed[toks]
    rms = lambda t, w: t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + cfg.rms_norm_eps) * w  # noqa: E731
    qkv = x @ L.wqkv.T
    H, KVH, D = 4, 2, 32
    q = rms(qkv[:, :H * D], L.q_norm).view(4, H, D)
    k = rms(qkv[:, H * D:(H + KVH) * D], L.k_norm).view(4, KVH, D)
    v = qkv[:, (H + KVH) * D:].view(4, KVH, D)
    from mlx_swift_lm_b200.ops.reference import apply_rope_ref, attention_rows_ref

    pos = torch.arange(4)
    q = apply_rope_ref(q, pos, m.cos_sin, m.rot_dim)
    k = apply_rope_ref(k, pos, m.cos_sin, m.rot_dim)
    a = attention_rows_ref(q, k, v, pos, 4, cfg.scale).reshape(4, H * D)
    h = x + rms(a @ L.wo.T, L.post_attn_norm)
    from mlx_swift_lm_b200.ops.reference import deinterleave_gate_up

    g, u = deinterleave_gate_up(L.wgu)
    mlp = (torch.nn.functional.silu(h @ g.T) * (h @ u.T)) @ L.wd.T
    out = rms(h + rms(mlp, L.post_ffn_norm), m.norm)
    torch.testing.assert_close(got, out, atol=2e-4, rtol=2e-4)


def test_apertus_xielu_mlp():
    from mlx_swift_lm_b200.ops.reference import xielu_ref

    cfg = build_config(_hf("apertus"))
    assert cfg.hidden_act == "xielu" and cfg.qk_norm and cfg.glu_epi == "xielu"
    m = _engine_vs_dense(cfg)
    L = m.layers[0]
    assert L.act_params.shape == (4,) and L.wgu.shape[0] == cfg.intermediate_size
    x = torch.linspace(-4, 4, 101)
    p = torch.tensor([0.3, -0.2, 0.5, -1e-6])
    y = xielu_ref(x, p)
    ap, an = torch.nn.functional.softplus(p[0]), 0.5 + torch.nn.functional.softplus(p[1])
    want = torch.where(x > 0, ap * x * x + 0.5 * x, an * (torch.exp(torch.clamp(x, max=-1e-6)) - 1) - an * x + 0.5 * x)
    torch.testing.assert_close(y, want)


def test_lfm2_moe_and_bailing_configs_run():
    cfg = build_config(_hf("lfm2_moe", num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                           num_dense_layers=1, use_expert_bias=True, routed_scaling_factor=2.0,
                           layer_types=["conv", "full_attention", "conv", "full_attention"], conv_L_cache=3))
    assert cfg.moe_layers == [False, True, True, True] and cfg.router_mode == "sigmoid_group"
    assert cfg.routed_scaling_factor == 2.0
    _engine_vs_dense(cfg)
    cfg = build_config(_hf("bailing_moe", num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                           first_k_dense_replace=1, num_shared_experts=1, use_qk_norm=True, n_group=2,
                           topk_group=1, partial_rotary_factor=0.5))
    assert cfg.qk_norm and cfg.shared_expert_intermediate_size == 64 and cfg.router_n_group == 2
    assert cfg.partial_rotary_factor == 0.5 and cfg.extra["fused_qkv"]
    _engine_vs_dense(cfg)


def test_family_name_maps():
    from mlx_swift_lm_b200.loader.load import _BAILING_RENAMES, _lfm2_names, _renamed

    t = _lfm2_names({"model.layers.2.feed_forward.experts.3.w1.weight": 1, "model.layers.2.feed_forward.gate.weight": 2,
                     "model.layers.2.feed_forward.expert_bias": 3, "model.layers.0.feed_forward.w2.weight": 4})
    assert set(t) == {"model.layers.2.mlp.experts.3.gate_proj.weight", "model.layers.2.mlp.gate.weight",
                      "model.layers.2.mlp.gate.e_score_correction_bias", "model.layers.0.mlp.down_proj.weight"}
    t = _renamed({"model.word_embeddings.weight": 0, "model.layers.0.attention.query_key_value.weight": 1,
                  "model.layers.0.attention.dense.weight": 2, "model.layers.1.mlp.gate.gate_proj.weight": 3,
                  "model.layers.1.mlp.gate.expert_bias": 4}, _BAILING_RENAMES)
    assert set(t) == {"model.embed_tokens.weight", "model.layers.0.self_attn.qkv_proj.weight",
                      "model.layers.0.self_attn.o_proj.weight", "model.layers.1.mlp.gate.weight",
                      "model.layers.1.mlp.gate.e_score_correction_bias"}
