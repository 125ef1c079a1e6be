"""Multi-head latent attention families (DeepSeek V2 / V3, GLM-4.7-Flash) on
CPU: config translation, one layer's attention against a direct restatement
of MLXLLM/Models/DeepseekV3.swift (attention at the unpadded head dims), the
paged engine against the dense path, the DeepSeek V2 group-limited greedy
gate, and checkpoint round trips (HF kv_b_proj and the MLX embed_q /
unembed_out split)."""
import math

import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models import mla
from mlx_swift_lm_b200.models.families import build_config
from mlx_swift_lm_b200.ops import moe as moe_ops


def _mla_hf(mt="deepseek_v3", **kw):
    d = dict(model_type=mt, vocab_size=300, hidden_size=96, num_hidden_layers=3, num_attention_heads=4,
             num_key_value_heads=4, intermediate_size=192, moe_intermediate_size=64, n_routed_experts=8,
             num_experts_per_tok=2, n_shared_experts=1, first_k_dense_replace=1, n_group=2, topk_group=1,
             routed_scaling_factor=1.5, norm_topk_prob=True, q_lora_rank=32, kv_lora_rank=48,
             qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32, rms_norm_eps=1e-6, rope_theta=10000.0,
             max_position_embeddings=4096, tie_word_embeddings=False,
             rope_scaling={"type": "yarn", "factor": 4.0, "original_max_position_embeddings": 512,
                           "beta_fast": 32, "beta_slow": 1, "mscale": 1.0, "mscale_all_dim": 1.0})
    d.update(kw)
    return d


def test_deepseek_mla_config_and_engine():
    cfg = build_config(_mla_hf())
    assert cfg.extra["mla"] and cfg.head_dim == 64 and cfg.num_kv_heads == 4
    assert cfg.rope_interleaved and round(cfg.partial_rotary_factor * 64) == 16
    m = 0.1 * math.log(4.0) + 1.0
    assert abs(cfg.scale - 48 ** -0.5 * m * m) < 1e-9
    assert cfg.router_mode == "sigmoid_group" and cfg.moe_layers == [False, True, True]
    model = DecoderLM(cfg, "cpu", torch.float32).init_random(0, std=0.2)
    L = model.layers[0]
    assert L.wqkv is None and L.mla_kv_b.shape == (4 * 64, 48) and L.wo.shape == (96, 4 * 32)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 23, 15)]
    eng = EngineV2(model, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4,
                                                                        prefill_chunk_size=9),
                                              max_model_len=128, use_cuda_graphs=False))
    out = eng.generate(prompts, max_tokens=5)
    for p, o in zip(prompts, out):
        cache = model.new_cache()
        logits = model.forward_dense(torch.tensor(p), cache)
        want = []
        for _ in range(5):
            t = int(logits[-1].argmax())
            want.append(t)
            logits = model.forward_dense(torch.tensor([t]), cache)
        assert o == want


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope_interleaved(x, pos, theta_inv, mscale):
    # x [T, ..., d] with pairs (2i, 2i+1) rotated by pos * inv[i]
    ang = pos[:, None].double() * theta_inv[None, :].double()
    while ang.dim() < x.dim():
        ang = ang[:, None]
    c, s = (ang.cos() * mscale).float(), (ang.sin() * mscale).float()
    x1, x2 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x1 * c - x2 * s
    out[..., 1::2] = x2 * c + x1 * s
    return out


@pytest.mark.parametrize("q_lora", [32, 0])
def test_mla_matches_direct_formula(q_lora):
    """Layer-0 attention output of the framework (zero-padded heads in the
    cache) equals the MLA formula at the true head dims."""
    hf = _mla_hf(q_lora_rank=q_lora or None, rope_scaling=None)
    cfg = build_config(hf)
    model = DecoderLM(cfg, "cpu", torch.float32).init_random(5, std=0.2)
    L = model.layers[0]
    T, H, eps = 11, 4, cfg.rms_norm_eps
    nope, rd, vd, kl = 32, 16, 32, 48
    x = torch.randn(T, 96, generator=torch.Generator().manual_seed(9))
    pos = torch.arange(T, dtype=torch.int32)
    got = mla.dense_attention(model, L, x, model.new_cache(), 0, pos)

    q = (_rms(x @ L.mla_q_a.T, L.mla_q_a_norm, eps) @ L.mla_q_b.T) if q_lora else x @ L.mla_q_b.T
    q = q.view(T, H, nope + rd)
    kva = x @ L.mla_kv_a.T
    c, kpe = kva[:, :kl], kva[:, kl:]
    kv = (_rms(c, L.mla_kv_a_norm, eps) @ L.mla_kv_b.T).view(T, H, nope + vd)
    inv = 1.0 / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float64) / rd))
    qpe = _rope_interleaved(q[..., nope:], pos, inv, 1.0)
    kpe = _rope_interleaved(kpe, pos, inv, 1.0)
    qf = torch.cat([q[..., :nope], qpe], -1)
    kf = torch.cat([kv[..., :nope], kpe[:, None, :].expand(T, H, rd)], -1)
    v = kv[..., nope:]
    s = torch.einsum("thd,shd->hts", qf, kf) * (nope + rd) ** -0.5
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    a = torch.einsum("hts,shd->thd", s.softmax(-1), v).reshape(T, H * vd)
    want = a @ L.wo.T
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()


def test_deepseek_v2_group_limited_greedy_gate():
    """softmax over all experts, groups ranked by their best probability,
    top-k among the kept groups, weights = probabilities times the routed
    scale, no renormalisation (MLXLLM/Models/DeepseekV2.swift:252-274)."""
    cfg = build_config(_mla_hf("deepseek_v2", topk_method="group_limited_greedy", n_group=4, topk_group=2,
                               norm_topk_prob=None, scoring_func="softmax"))
    assert cfg.router_mode == "softmax_topk" and not cfg.norm_topk_prob and cfg.router_n_group == 4
    greedy = build_config(_mla_hf("deepseek_v2", topk_method="greedy", n_group=4, topk_group=2))
    assert greedy.router_n_group == 1
    torch.manual_seed(1)
    E, k, G, TG = 32, 6, 4, 2
    lg = torch.randn(25, E) * 2
    w, idx = moe_ops.route_topk(lg, k, "softmax_topk", False, None, G, TG, 2.0)
    p = lg.double().softmax(-1)
    for t in range(lg.shape[0]):
        gmax = [p[t, g * 8:(g + 1) * 8].max().item() for g in range(G)]
        keep = sorted(range(G), key=lambda g: (-gmax[g], g))[:TG]
        masked = [p[t, e].item() if e // 8 in keep else 0.0 for e in range(E)]
        order = sorted(range(E), key=lambda e: (-masked[e], e))[:k]
        assert idx[t].tolist() == order
        assert torch.allclose(w[t], torch.tensor([masked[e] * 2.0 for e in order], dtype=torch.float32),
                              atol=1e-6)


def test_deepseek_v2_rejects_sigmoid_scoring():
    with pytest.raises(NotImplementedError):
        build_config(_mla_hf("deepseek_v2", scoring_func="sigmoid"))


@pytest.mark.parametrize("mlx_split", [False, True])
def test_mla_checkpoint_roundtrip(tmp_path, mlx_split):
    from safetensors.torch import load_file, save_file

    from mlx_swift_lm_b200.loader.convert import save_model
    from mlx_swift_lm_b200.loader.load import load_model

    cfg = build_config(_mla_hf("glm4_moe_lite"))
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(4, std=0.2)
    d = tmp_path / "mla"
    save_model(m, str(d), dtype=torch.float32)
    if mlx_split:  # rewrite kv_b_proj as the per-head embed_q / unembed_out pair
        import glob

        for f in glob.glob(str(d / "*.safetensors")):
            t = load_file(f)
            for key in [k for k in t if k.endswith("kv_b_proj.weight")]:
                w = t.pop(key).view(4, 32 + 32, 48)
                base = key[:-len("kv_b_proj.weight")]
                t[base + "embed_q.weight"] = w[:, :32, :].transpose(1, 2).contiguous()
                t[base + "unembed_out.weight"] = w[:, 32:, :].contiguous()
            save_file(t, f)
    m2, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert m2.cfg.extra["mla"] and m2.cfg.head_dim == 64
    toks = torch.arange(3, 30)
    assert torch.allclose(m2.forward_dense(toks, m2.new_cache()), m.forward_dense(toks, m.new_cache()), atol=1e-4)
