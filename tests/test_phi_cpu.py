"""Phi-2 (parallel attention + MLP block, LayerNorm with bias, partial
rotary, biased projections and head) on CPU: HF-named checkpoints load with
logits equal to a direct re-statement of MLXLLM/Models/Phi.swift, and the
paged engine matches the dense forward."""
import json
import math

import torch

from mlx_swift_lm_b200 import EngineConfig, EngineV2, SchedulerConfig

HF = {"model_type": "phi", "vocab_size": 300, "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 4,
      "num_key_value_heads": 4, "intermediate_size": 128, "partial_rotary_factor": 0.5, "layer_norm_eps": 1e-5,
      "rope_theta": 10000.0, "max_position_embeddings": 2048, "tie_word_embeddings": False}


def _tensors(seed=0):
    g = torch.Generator().manual_seed(seed)

    def rn(*s, std=0.2):
        return torch.randn(*s, generator=g) * std

    t = {"model.embed_tokens.weight": rn(300, 64, std=0.5), "model.final_layernorm.weight": 1 + rn(64),
         "model.final_layernorm.bias": rn(64), "lm_head.weight": rn(300, 64), "lm_head.bias": rn(300)}
    for i in range(2):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"], t[p + "input_layernorm.bias"] = 1 + rn(64), rn(64)
        for n in ("q_proj", "k_proj", "v_proj", "dense"):
            t[p + f"self_attn.{n}.weight"], t[p + f"self_attn.{n}.bias"] = rn(64, 64), rn(64)
        t[p + "mlp.fc1.weight"], t[p + "mlp.fc1.bias"] = rn(128, 64), rn(128)
        t[p + "mlp.fc2.weight"], t[p + "mlp.fc2.bias"] = rn(64, 128), rn(64)
    return t


def _rope_partial(x, pos, rot, base):
    inv = 1.0 / (base ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    ang = (pos[:, None].double() * inv[None]).float()
    c, s = ang.cos()[:, None], ang.sin()[:, None]
    xr, xp = x[..., :rot], x[..., rot:]
    x1, x2 = xr[..., :rot // 2], xr[..., rot // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s, xp], -1)


def direct_forward(t, ids):
    T = ids.shape[0]
    ln = torch.nn.functional.layer_norm
    x = t["model.embed_tokens.weight"][ids]
    pos = torch.arange(T)
    for i in range(2):
        p = f"model.layers.{i}."
        h = ln(x, (64,), t[p + "input_layernorm.weight"], t[p + "input_layernorm.bias"], 1e-5)

        def lin(n, v):
            return v @ t[p + n + ".weight"].t() + t[p + n + ".bias"]

        q = _rope_partial(lin("self_attn.q_proj", h).reshape(T, 4, 16), pos, 8, 10000.0)
        k = _rope_partial(lin("self_attn.k_proj", h).reshape(T, 4, 16), pos, 8, 10000.0)
        v = lin("self_attn.v_proj", h).reshape(T, 4, 16)
        s = torch.einsum("thd,shd->hts", q, k) / 4.0
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -math.inf)
        a = lin("self_attn.dense", torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, -1))
        f = lin("mlp.fc2", torch.nn.functional.gelu(lin("mlp.fc1", h), approximate="tanh"))
        x = x + a + f
    x = ln(x, (64,), t["model.final_layernorm.weight"], t["model.final_layernorm.bias"], 1e-5)
    return x @ t["lm_head.weight"].t() + t["lm_head.bias"]


def test_phi_checkpoint_and_engine(tmp_path):
    from mlx_swift_lm_b200.loader.convert import write_shards
    from mlx_swift_lm_b200.loader.load import load_model

    t = _tensors()
    d = tmp_path / "phi"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(HF))
    write_shards(t, str(d))
    m, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert m.cfg.parallel_block and m.rot_dim == 8
    ids = torch.arange(3, 25)
    got = m.forward_dense(ids, m.new_cache())
    want = direct_forward(t, ids)
    assert torch.allclose(got, want, atol=2e-3, rtol=1e-3), (got - want).abs().max()
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 300, (n,), generator=g).tolist() for n in (5, 19)]
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
