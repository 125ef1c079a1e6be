"""LFM2 (gated short-conv / attention hybrid) on CPU: the short-conv oracle
is exact under chunking, HF-named checkpoints load with logits equal to a
direct re-statement of MLXLLM/Models/LFM2.swift, and the paged engine with
conv-state slots matches the dense forward."""
import json
import math

import torch

from mlx_swift_lm_b200 import EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.ops import reference as ref

HF = {"model_type": "lfm2", "vocab_size": 300, "hidden_size": 64, "num_hidden_layers": 4, "num_attention_heads": 4,
      "num_key_value_heads": 2, "max_position_embeddings": 4096, "norm_eps": 1e-5, "conv_bias": False,
      "conv_L_cache": 3, "block_ff_dim": 192, "block_multiple_of": 64, "block_auto_adjust_ff_dim": True,
      "layer_types": ["conv", "conv", "full_attention", "conv"], "rope_theta": 1000000.0,
      "tie_word_embeddings": True}
FF = 128  # int(2 * 192 / 3) rounded up to 64


def test_short_conv_chunking_is_exact():
    torch.manual_seed(0)
    C, T = 16, 11
    P = torch.randn(T, 3 * C)
    w, b = torch.randn(C, 3), torch.randn(C)
    cs = torch.zeros(1, 2, C)
    whole = ref.short_conv_ref(P, [0, T], [1], [0], cs, w, b)
    cs2 = torch.zeros(1, 2, C)
    parts = [ref.short_conv_ref(P[a:c], [0, c - a], [1 if a == 0 else 0], [0], cs2, w, b)
             for a, c in [(0, 1), (1, 2), (2, 7), (7, 11)]]
    assert torch.allclose(torch.cat(parts), whole, atol=1e-6) and torch.equal(cs, cs2)


def _tensors(seed=0):
    g = torch.Generator().manual_seed(seed)

    def rn(*s, std=0.2):
        return torch.randn(*s, generator=g) * std

    t = {"model.embed_tokens.weight": rn(300, 64, std=0.5), "model.embedding_norm.weight": 1 + rn(64)}
    for i, kind in enumerate(HF["layer_types"]):
        p = f"model.layers.{i}."
        t[p + "operator_norm.weight"], t[p + "ffn_norm.weight"] = 1 + rn(64), 1 + rn(64)
        if kind == "conv":
            t[p + "conv.in_proj.weight"], t[p + "conv.out_proj.weight"] = rn(192, 64), rn(64, 64)
            t[p + "conv.conv.weight"] = rn(64, 1, 3, std=0.5)
        else:
            a = p + "self_attn."
            t[a + "q_proj.weight"], t[a + "k_proj.weight"] = rn(64, 64), rn(32, 64)
            t[a + "v_proj.weight"], t[a + "out_proj.weight"] = rn(32, 64), rn(64, 64)
            t[a + "q_layernorm.weight"], t[a + "k_layernorm.weight"] = 1 + rn(16), 1 + rn(16)
        t[p + "feed_forward.w1.weight"], t[p + "feed_forward.w3.weight"] = rn(FF, 64), rn(FF, 64)
        t[p + "feed_forward.w2.weight"] = rn(64, FF)
    return t


def _rms(x, w, eps=1e-5):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, base):
    d = x.shape[-1]
    inv = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = (pos[:, None].double() * inv[None]).float()
    c, s = ang.cos()[:, None], ang.sin()[:, None]
    x1, x2 = x[..., :d // 2], x[..., d // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def direct_forward(t, ids):
    T = ids.shape[0]
    x = t["model.embed_tokens.weight"][ids]
    pos = torch.arange(T)
    for i, kind in enumerate(HF["layer_types"]):
        p = f"model.layers.{i}."
        h = _rms(x, t[p + "operator_norm.weight"])
        if kind == "conv":
            bcx = h @ t[p + "conv.in_proj.weight"].t()
            B, Cg, xx = bcx[:, :64], bcx[:, 64:128], bcx[:, 128:]
            bx = torch.cat([torch.zeros(2, 64), B * xx])
            w = t[p + "conv.conv.weight"][:, 0, :]
            conv = sum(w[:, j] * bx[j:j + T] for j in range(3))
            d = (Cg * conv) @ t[p + "conv.out_proj.weight"].t()
        else:
            a = p + "self_attn."
            q = _rms((h @ t[a + "q_proj.weight"].t()).reshape(T, 4, 16), t[a + "q_layernorm.weight"])
            k = _rms((h @ t[a + "k_proj.weight"].t()).reshape(T, 2, 16), t[a + "k_layernorm.weight"])
            v = (h @ t[a + "v_proj.weight"].t()).reshape(T, 2, 16)
            q, k = _rope(q, pos, HF["rope_theta"]), _rope(k, pos, HF["rope_theta"])
            k, v = k.repeat_interleave(2, 1), v.repeat_interleave(2, 1)
            s = torch.einsum("thd,shd->hts", q, k) / 4.0
            s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -math.inf)
            d = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, -1) @ t[a + "out_proj.weight"].t()
        x = x + d
        h = _rms(x, t[p + "ffn_norm.weight"])
        f = torch.nn.functional.silu(h @ t[p + "feed_forward.w1.weight"].t()) * (h @ t[p + "feed_forward.w3.weight"].t())
        x = x + f @ t[p + "feed_forward.w2.weight"].t()
    return _rms(x, t["model.embedding_norm.weight"]) @ t["model.embed_tokens.weight"].t()


def test_lfm2_checkpoint_and_engine(tmp_path):
    from mlx_swift_lm_b200.loader.convert import write_shards
    from mlx_swift_lm_b200.loader.load import load_model

    t = _tensors()
    d = tmp_path / "lfm2"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(HF))
    write_shards(t, str(d))
    m, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert m.cfg.intermediate_size == FF and m.num_kv_layers == 1
    ids = torch.arange(3, 25)
    got = m.forward_dense(ids, m.new_cache())
    want = direct_forward(t, ids)
    assert torch.allclose(got, want, atol=2e-3, rtol=1e-3), (got - want).abs().max()
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 300, (n,), generator=g).tolist() for n in (5, 19, 12)]
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=7),
                                          max_model_len=128, use_cuda_graphs=False))
    out = eng.generate(prompts, max_tokens=6)
    for p, o in zip(prompts, out):
        cache = m.new_cache()
        logits = m.forward_dense(torch.tensor(p), cache)
        want_t = []
        for _ in range(6):
            tk = int(logits[-1].argmax())
            want_t.append(tk)
            logits = m.forward_dense(torch.tensor([tk]), cache)
        assert o == want_t
