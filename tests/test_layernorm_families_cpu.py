"""LayerNorm families on CPU: Cohere (parallel attention + SwiGLU under one
LayerNorm, logit scale) and StarCoder2 (LayerNorm with bias, biased GELU
MLP) load HF-named tensors with logits equal to a direct re-statement; the
refused architectures fail loudly instead of loading wrongly."""
import json
import math

import pytest
import torch

from mlx_swift_lm_b200.models.families import build_config


def _rope(x, pos, base=10000.0):
    d = x.shape[-1]
    inv = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = (pos[:, None].double() * inv[None]).float()
    c, s = ang.cos()[:, None], ang.sin()[:, None]
    x1, x2 = x[..., :d // 2], x[..., d // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def _attn(t, a, h, T, bias):
    def lin(n):
        y = h @ t[a + n + ".weight"].t()
        return y + t[a + n + ".bias"] if bias else y

    pos = torch.arange(T)
    q, k, v = (lin(n).reshape(T, 4, 16) for n in ("q_proj", "k_proj", "v_proj"))
    q, k = _rope(q, pos), _rope(k, pos)
    s = torch.einsum("thd,shd->hts", q, k) / 4.0
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -math.inf)
    o = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, -1) @ t[a + "o_proj.weight"].t()
    return o + t[a + "o_proj.bias"] if bias else o


def _make(kind, seed=0):
    g = torch.Generator().manual_seed(seed)

    def rn(*s, std=0.2):
        return torch.randn(*s, generator=g) * std

    bias = kind == "starcoder2"
    t = {"model.embed_tokens.weight": rn(200, 64, std=0.5), "model.norm.weight": 1 + rn(64)}
    if bias:
        t["model.norm.bias"] = rn(64)
        t["lm_head.weight"] = rn(200, 64)
    for i in range(2):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = 1 + rn(64)
        if bias:
            t[p + "input_layernorm.bias"] = rn(64)
            t[p + "post_attention_layernorm.weight"], t[p + "post_attention_layernorm.bias"] = 1 + rn(64), rn(64)
        for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
            t[p + f"self_attn.{n}.weight"] = rn(64, 64)
            if bias:
                t[p + f"self_attn.{n}.bias"] = rn(64)
        if bias:
            t[p + "mlp.c_fc.weight"], t[p + "mlp.c_fc.bias"] = rn(128, 64), rn(128)
            t[p + "mlp.c_proj.weight"], t[p + "mlp.c_proj.bias"] = rn(64, 128), rn(64)
        else:
            t[p + "mlp.gate_proj.weight"], t[p + "mlp.up_proj.weight"] = rn(128, 64), rn(128, 64)
            t[p + "mlp.down_proj.weight"] = rn(64, 128)
    return t


def _direct(t, kind, ids):
    T = ids.shape[0]
    ln = torch.nn.functional.layer_norm
    bias = kind == "starcoder2"
    x = t["model.embed_tokens.weight"][ids]
    for i in range(2):
        p = f"model.layers.{i}."
        h = ln(x, (64,), t[p + "input_layernorm.weight"], t.get(p + "input_layernorm.bias"), 1e-5)
        a = _attn(t, p + "self_attn.", h, T, bias)
        if kind == "cohere":
            m = (torch.nn.functional.silu(h @ t[p + "mlp.gate_proj.weight"].t()) * (h @ t[p + "mlp.up_proj.weight"].t())
                 ) @ t[p + "mlp.down_proj.weight"].t()
            x = x + a + m
        else:
            x = x + a
            h = ln(x, (64,), t[p + "post_attention_layernorm.weight"], t[p + "post_attention_layernorm.bias"], 1e-5)
            f = torch.nn.functional.gelu(h @ t[p + "mlp.c_fc.weight"].t() + t[p + "mlp.c_fc.bias"], approximate="tanh")
            x = x + f @ t[p + "mlp.c_proj.weight"].t() + t[p + "mlp.c_proj.bias"]
    x = ln(x, (64,), t["model.norm.weight"], t.get("model.norm.bias"), 1e-5)
    if kind == "cohere":
        return (x @ t["model.embed_tokens.weight"].t()) * 0.25
    return x @ t["lm_head.weight"].t()


@pytest.mark.parametrize("kind", ["cohere", "starcoder2"])
def test_layernorm_family_matches_direct(tmp_path, kind):
    from mlx_swift_lm_b200.loader.convert import write_shards
    from mlx_swift_lm_b200.loader.load import load_model

    hf = {"model_type": kind, "vocab_size": 200, "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 4,
          "num_key_value_heads": 4, "intermediate_size": 128, "layer_norm_eps": 1e-5, "norm_epsilon": 1e-5,
          "rope_theta": 10000.0, "max_position_embeddings": 2048, "logit_scale": 0.25,
          "hidden_act": "gelu_pytorch_tanh" if kind == "starcoder2" else "silu",
          "tie_word_embeddings": kind == "cohere", "use_bias": True}
    t = _make(kind)
    d = tmp_path / kind
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hf))
    write_shards(t, str(d))
    m, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    ids = torch.arange(3, 20)
    got = m.forward_dense(ids, m.new_cache())
    want = _direct(t, kind, ids)
    assert torch.allclose(got, want, atol=2e-3, rtol=1e-3), (got - want).abs().max()


def test_refused_architectures():
    """Variants outside what the families serve fail at config time."""
    with pytest.raises(NotImplementedError):
        build_config({"model_type": "cohere", "vocab_size": 10, "hidden_size": 8, "num_hidden_layers": 1,
                      "num_attention_heads": 1, "use_qk_norm": True})
    with pytest.raises(NotImplementedError):
        build_config({"model_type": "deepseek_v2", "vocab_size": 10, "hidden_size": 8, "num_hidden_layers": 1,
                      "num_attention_heads": 1, "kv_lora_rank": 8, "qk_nope_head_dim": 8, "qk_rope_head_dim": 4,
                      "v_head_dim": 8, "scoring_func": "sigmoid"})
