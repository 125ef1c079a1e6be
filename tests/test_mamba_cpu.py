"""Mamba-2 mixers (NemotronH hybrids, pure Mamba-2) on CPU: the fp32 layer
oracle is exact under chunking, the paged engine with recurrent-state slots
matches the dense forward, and HF-named checkpoints load into the fused
layout (reordered in-projection and conv channels) with logits equal to a
direct re-statement of the HF / mlx-lm forward."""
import json
import math

import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.families import build_config
from mlx_swift_lm_b200.ops import reference as ref

NH = {"model_type": "nemotron_h", "vocab_size": 300, "hidden_size": 64, "num_hidden_layers": 5,
      "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16, "mamba_num_heads": 8, "mamba_head_dim": 16,
      "ssm_state_size": 32, "n_groups": 2, "conv_kernel": 4, "intermediate_size": 96,
      "hybrid_override_pattern": "M-M*-", "layer_norm_epsilon": 1e-5, "use_conv_bias": True,
      "time_step_limit": [0.0, 2.0], "tie_word_embeddings": False}
M2 = {"model_type": "mamba2", "vocab_size": 300, "hidden_size": 64, "num_hidden_layers": 3, "num_heads": 8,
      "head_dim": 16, "state_size": 32, "n_groups": 1, "conv_kernel": 4, "layer_norm_epsilon": 1e-5,
      "use_conv_bias": True, "tie_word_embeddings": True}


def test_mamba_ref_chunking_is_exact():
    torch.manual_seed(0)
    G, N, H, Pd = 2, 16, 4, 8
    C = 2 * G * N + H * Pd
    T = 13
    P = torch.randn(T, C + H * Pd + H)
    conv_w, conv_b = torch.randn(C, 4) * 0.5, torch.randn(C) * 0.1
    A_log, dt_bias, D = torch.rand(H), torch.randn(H), torch.randn(H)
    norm_w = torch.rand(H * Pd) + 0.5
    args = (conv_w, conv_b, A_log, dt_bias, D, norm_w, G, N, H, Pd, 1e-5, H * Pd // G, (0.0, 3.0))

    def fresh():
        return torch.zeros(1, 3, C), torch.zeros(1, H, Pd, N)

    cs, ss = fresh()
    whole = ref.mamba_layer_ref(P, [0, T], [1], [0], cs, ss, *args)
    cs2, ss2 = fresh()
    parts = [ref.mamba_layer_ref(P[a:b], [0, b - a], [1 if a == 0 else 0], [0], cs2, ss2, *args)
             for a, b in [(0, 2), (2, 3), (3, 10), (10, 13)]]
    assert torch.allclose(torch.cat(parts), whole, atol=1e-5)
    assert torch.allclose(ss2, ss, atol=1e-6) and torch.equal(cs2, cs)


@pytest.mark.parametrize("hf", [NH, M2])
def test_engine_matches_dense_forward(hf):
    cfg = build_config(hf)
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(1, std=0.2)
    assert [L.block for L in m.layers] == cfg.layer_blocks
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 19, 12)]
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=7),
                                          max_model_len=128, use_cuda_graphs=False))
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
    assert eng.kv.rec.num_free == 4


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def hf_forward(t, hf, ids):
    """Direct re-statement of the NemotronH / Mamba-2 forward on HF-named
    tensors (single sequence, from position 0)."""
    nemo = hf["model_type"] == "nemotron_h"
    eps = hf["layer_norm_epsilon"]
    x = t["backbone.embeddings.weight"][ids]
    T = x.shape[0]
    pat = hf.get("hybrid_override_pattern") or "M" * hf["num_hidden_layers"]
    H = hf["mamba_num_heads"] if nemo else hf["num_heads"]
    Pd = hf["mamba_head_dim"] if nemo else hf["head_dim"]
    N = hf["ssm_state_size"] if nemo else hf["state_size"]
    G = hf["n_groups"]
    I = H * Pd
    lo, hi = hf.get("time_step_limit", [0.0, math.inf])
    for i, c in enumerate(pat):
        p = f"backbone.layers.{i}."
        h = _rms(x, t[p + "norm.weight"], eps)
        mx = p + "mixer."
        if c == "M":
            zxbcdt = h @ t[mx + "in_proj.weight"].t()
            z, xBC, dt = zxbcdt[:, :I], zxbcdt[:, I:2 * I + 2 * G * N], zxbcdt[:, 2 * I + 2 * G * N:]
            w = t[mx + "conv1d.weight"][:, 0, :]  # [C, K]
            pad = torch.cat([torch.zeros(3, xBC.shape[1]), xBC])
            conv = sum(w[:, j] * pad[j:j + T] for j in range(4)) + t[mx + "conv1d.bias"]
            conv = conv * torch.sigmoid(conv)
            xs, Bm, Cm = conv[:, :I].reshape(T, H, Pd), conv[:, I:I + G * N].reshape(T, G, N), \
                conv[:, I + G * N:].reshape(T, G, N)
            dt = torch.nn.functional.softplus(dt + t[mx + "dt_bias"]).clamp(lo, hi)
            A = -torch.exp(t[mx + "A_log"])
            S = torch.zeros(H, Pd, N)
            ys = []
            for k in range(T):
                Bh = Bm[k].repeat_interleave(H // G, 0)
                Ch = Cm[k].repeat_interleave(H // G, 0)
                S = S * torch.exp(A * dt[k])[:, None, None] + (xs[k] * dt[k][:, None])[:, :, None] * Bh[:, None, :]
                ys.append((S * Ch[:, None, :]).sum(-1) + t[mx + "D"][:, None] * xs[k])
            y = torch.stack(ys).reshape(T, I) * torch.nn.functional.silu(z)
            gsz = I // G if nemo else I
            yg = y.reshape(T, -1, gsz)
            y = (yg * torch.rsqrt(yg.pow(2).mean(-1, keepdim=True) + eps)).reshape(T, I) * t[mx + "norm.weight"]
            x = x + y @ t[mx + "out_proj.weight"].t()
        elif c == "*":
            nh, kvh, hd = hf["num_attention_heads"], hf["num_key_value_heads"], hf["head_dim"]
            q = (h @ t[mx + "q_proj.weight"].t()).reshape(T, nh, hd)
            k = (h @ t[mx + "k_proj.weight"].t()).reshape(T, kvh, hd).repeat_interleave(nh // kvh, 1)
            v = (h @ t[mx + "v_proj.weight"].t()).reshape(T, kvh, hd).repeat_interleave(nh // kvh, 1)
            s = torch.einsum("thd,shd->hts", q, k) / math.sqrt(hd)
            s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -math.inf)
            a = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, -1)
            x = x + a @ t[mx + "o_proj.weight"].t()
        else:
            u = torch.relu(h @ t[mx + "up_proj.weight"].t()).square()
            x = x + u @ t[mx + "down_proj.weight"].t()
    x = _rms(x, t["backbone.norm_f.weight"], eps)
    head = t.get("lm_head.weight", t["backbone.embeddings.weight"])
    return x @ head.t()


def _hf_tensors(hf, seed=0):
    g = torch.Generator().manual_seed(seed)
    nemo = hf["model_type"] == "nemotron_h"

    def rn(*s, std=0.2):
        return torch.randn(*s, generator=g) * std

    Hd = hf["hidden_size"]
    H = hf["mamba_num_heads"] if nemo else hf["num_heads"]
    Pd = hf["mamba_head_dim"] if nemo else hf["head_dim"]
    N = hf["ssm_state_size"] if nemo else hf["state_size"]
    G = hf["n_groups"]
    I = H * Pd
    C = I + 2 * G * N
    t = {"backbone.embeddings.weight": rn(hf["vocab_size"], Hd, std=0.5), "backbone.norm_f.weight": 1 + rn(Hd)}
    if not hf.get("tie_word_embeddings"):
        t["lm_head.weight"] = rn(hf["vocab_size"], Hd)
    pat = hf.get("hybrid_override_pattern") or "M" * hf["num_hidden_layers"]
    for i, c in enumerate(pat):
        p = f"backbone.layers.{i}."
        t[p + "norm.weight"] = 1 + rn(Hd)
        mx = p + "mixer."
        if c == "M":
            t[mx + "in_proj.weight"] = rn(2 * I + 2 * G * N + H, Hd)
            t[mx + "conv1d.weight"] = rn(C, 1, 4, std=0.5)
            t[mx + "conv1d.bias"] = rn(C, std=0.1)
            t[mx + "A_log"] = torch.rand(H, generator=g) * 2
            t[mx + "dt_bias"] = rn(H)
            t[mx + "D"] = 1 + rn(H)
            t[mx + "norm.weight"] = 1 + rn(I)
            t[mx + "out_proj.weight"] = rn(Hd, I)
        elif c == "*":
            nh, kvh, hd = hf["num_attention_heads"], hf["num_key_value_heads"], hf["head_dim"]
            t[mx + "q_proj.weight"], t[mx + "k_proj.weight"] = rn(nh * hd, Hd), rn(kvh * hd, Hd)
            t[mx + "v_proj.weight"], t[mx + "o_proj.weight"] = rn(kvh * hd, Hd), rn(Hd, nh * hd)
        else:
            t[mx + "up_proj.weight"], t[mx + "down_proj.weight"] = rn(hf["intermediate_size"], Hd), \
                rn(Hd, hf["intermediate_size"])
    return t


@pytest.mark.parametrize("hf", [NH, M2])
def test_hf_checkpoint_matches_direct_forward(tmp_path, hf):
    from mlx_swift_lm_b200.loader.convert import write_shards
    from mlx_swift_lm_b200.loader.load import load_model

    t = _hf_tensors(hf)
    d = tmp_path / hf["model_type"]
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hf))
    write_shards(t, str(d))
    m, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    ids = torch.arange(7, 30) % hf["vocab_size"]
    got = m.forward_dense(ids, m.new_cache())
    want = hf_forward(t, hf, ids)
    assert torch.allclose(got, want, atol=2e-3, rtol=1e-3), (got - want).abs().max()


def test_dt_limit_resolution():
    from mlx_swift_lm_b200.models.families import _ssm_dt_limits

    assert _ssm_dt_limits({"time_step_limit": [0.0, 5.0]}) == (0.0, 5.0)
    assert _ssm_dt_limits({"time_step_limit": [0.5]}) == (0.5, 0.5)
    assert _ssm_dt_limits({"time_step_min": 0.001, "time_step_max": 0.1}) == (0.001, 0.1)
    assert _ssm_dt_limits({}) == (0.0, math.inf)
    with pytest.raises(ValueError):
        _ssm_dt_limits({"time_step_limit": [2.0, 1.0]})
