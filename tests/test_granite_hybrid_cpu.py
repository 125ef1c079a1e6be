"""Granite 4 hybrids (GraniteMoeHybrid) on CPU: HF-named tensors load into
the fused layout (Mamba-2 mixers, attention without rotation, top-k-softmax
experts from ``input_linear`` / ``output_linear``, shared MLP) with the
embedding / attention / residual / logits multipliers, and the logits equal
a direct re-statement of the forward (MLXLLM/Models/GraniteMoeHybrid.swift)."""
import json
import math

import torch

HF = {"model_type": "granitemoehybrid", "vocab_size": 320, "hidden_size": 64, "intermediate_size": 64,
      "num_hidden_layers": 3, "max_position_embeddings": 4096, "num_attention_heads": 4, "num_key_value_heads": 2,
      "attention_bias": False, "embedding_multiplier": 12.0, "attention_multiplier": 0.015625,
      "logits_scaling": 8.0, "residual_multiplier": 0.22, "layer_types": ["mamba", "attention", "mamba"],
      "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "num_local_experts": 4, "num_experts_per_tok": 2,
      "shared_intermediate_size": 64, "mamba_n_heads": 8, "mamba_d_head": 16, "mamba_d_state": 64,
      "mamba_d_conv": 4, "mamba_n_groups": 1, "mamba_conv_bias": True, "mamba_proj_bias": False,
      "position_embedding_type": "nope", "time_step_limit": [0.0, 10.0], "tie_word_embeddings": True}


def _rms(x, w, eps=1e-5):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _tensors(seed=0):
    g = torch.Generator().manual_seed(seed)

    def rn(*s, std=0.2):
        return torch.randn(*s, generator=g) * std

    Hd, H, P, N, G = 64, 8, 16, 64, 1
    I, C = H * P, H * P + 2 * G * N
    t = {"model.embed_tokens.weight": rn(320, Hd, std=0.1), "model.norm.weight": 1 + rn(Hd)}
    for i, kind in enumerate(HF["layer_types"]):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"], t[p + "post_attention_layernorm.weight"] = 1 + rn(Hd), 1 + rn(Hd)
        if kind == "mamba":
            m = p + "mamba."
            t[m + "in_proj.weight"] = rn(2 * I + 2 * G * N + H, Hd)
            t[m + "conv1d.weight"], t[m + "conv1d.bias"] = rn(C, 1, 4, std=0.5), rn(C, std=0.1)
            t[m + "A_log"], t[m + "dt_bias"], t[m + "D"] = torch.rand(H, generator=g), rn(H), 1 + rn(H)
            t[m + "norm.weight"], t[m + "out_proj.weight"] = 1 + rn(I), rn(Hd, I)
        else:
            a = p + "self_attn."
            t[a + "q_proj.weight"], t[a + "k_proj.weight"] = rn(64, Hd), rn(32, Hd)
            t[a + "v_proj.weight"], t[a + "o_proj.weight"] = rn(32, Hd), rn(Hd, 64)
        b = p + "block_sparse_moe."
        t[b + "router.layer.weight"] = rn(4, Hd)
        t[b + "input_linear.weight"], t[b + "output_linear.weight"] = rn(4, 128, Hd), rn(4, Hd, 64)
        t[p + "shared_mlp.input_linear.weight"], t[p + "shared_mlp.output_linear.weight"] = rn(128, Hd), rn(Hd, 64)
    return t


def direct_forward(t, ids):
    T = ids.shape[0]
    x = t["model.embed_tokens.weight"][ids] * HF["embedding_multiplier"]
    H, P, N, G = 8, 16, 64, 1
    I = H * P
    rm = HF["residual_multiplier"]
    for i, kind in enumerate(HF["layer_types"]):
        p = f"model.layers.{i}."
        h = _rms(x, t[p + "input_layernorm.weight"])
        if kind == "mamba":
            m = p + "mamba."
            zx = h @ t[m + "in_proj.weight"].t()
            z, xBC, dt = zx[:, :I], zx[:, I:2 * I + 2 * G * N], zx[:, 2 * I + 2 * G * N:]
            w = t[m + "conv1d.weight"][:, 0, :]
            pad = torch.cat([torch.zeros(3, xBC.shape[1]), xBC])
            cv = sum(w[:, j] * pad[j:j + T] for j in range(4)) + t[m + "conv1d.bias"]
            cv = cv * torch.sigmoid(cv)
            xs, Bm, Cm = cv[:, :I].reshape(T, H, P), cv[:, I:I + N], cv[:, I + N:]
            dt = torch.nn.functional.softplus(dt + t[m + "dt_bias"]).clamp(0.0, 10.0)
            A = -torch.exp(t[m + "A_log"])
            S = torch.zeros(H, P, N)
            ys = []
            for k in range(T):
                S = S * torch.exp(A * dt[k])[:, None, None] + (xs[k] * dt[k][:, None])[:, :, None] * Bm[k][None, None]
                ys.append((S * Cm[k][None, None]).sum(-1) + t[m + "D"][:, None] * xs[k])
            y = torch.stack(ys).reshape(T, I) * torch.nn.functional.silu(z)
            y = _rms(y, t[m + "norm.weight"])
            d = y @ t[m + "out_proj.weight"].t()
        else:
            a = p + "self_attn."
            q = (h @ t[a + "q_proj.weight"].t()).reshape(T, 4, 16)
            k = (h @ t[a + "k_proj.weight"].t()).reshape(T, 2, 16).repeat_interleave(2, 1)
            v = (h @ t[a + "v_proj.weight"].t()).reshape(T, 2, 16).repeat_interleave(2, 1)
            s = torch.einsum("thd,shd->hts", q, k) * HF["attention_multiplier"]
            s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -math.inf)
            d = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, -1) @ t[a + "o_proj.weight"].t()
        x = x + d * rm
        h = _rms(x, t[p + "post_attention_layernorm.weight"])
        b = p + "block_sparse_moe."
        lg = h @ t[b + "router.layer.weight"].t()
        tv, ti = torch.topk(lg, 2, dim=-1)
        gw = torch.softmax(tv, -1)
        out = torch.zeros_like(h)
        for r in range(T):
            for j in range(2):
                e = int(ti[r, j])
                gu = t[b + "input_linear.weight"][e] @ h[r]
                out[r] += gw[r, j] * (t[b + "output_linear.weight"][e] @ (torch.nn.functional.silu(gu[:64]) * gu[64:]))
        su = h @ t[p + "shared_mlp.input_linear.weight"].t()
        out = out + (torch.nn.functional.silu(su[:, :64]) * su[:, 64:]) @ t[p + "shared_mlp.output_linear.weight"].t()
        x = x + out * rm
    x = _rms(x, t["model.norm.weight"])
    return (x @ t["model.embed_tokens.weight"].t()) / HF["logits_scaling"]


def test_granite_hybrid_checkpoint_matches_direct_forward(tmp_path):
    from mlx_swift_lm_b200.loader.convert import write_shards
    from mlx_swift_lm_b200.loader.load import load_model

    t = _tensors()
    d = tmp_path / "g4"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(HF))
    write_shards(t, str(d))
    m, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert m.cfg.router_mode == "topk_softmax" and m.cfg.linear_kind == "mamba2" and m.rot_dim == 0
    assert m.lm_head is not m.embed  # logits divisor folded into an untied head
    ids = torch.arange(5, 26)
    got = m.forward_dense(ids, m.new_cache())
    want = direct_forward(t, ids)
    assert torch.allclose(got, want, atol=2e-3, rtol=1e-3), (got - want).abs().max()
