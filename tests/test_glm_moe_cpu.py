"""GLM-4.5-style MoE (sigmoid scores, group-limited corrected selection,
routed scaling, shared experts after dense layers) on CPU: the router
against a direct re-statement of MLXLLM/Models/GLM4MOE.swift:147-180, the
engine against the dense forward, and a checkpoint round trip."""
import copy

import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.families import build_config
from mlx_swift_lm_b200.ops import moe as moe_ops

HF = {"model_type": "glm4_moe", "vocab_size": 400, "hidden_size": 128, "num_hidden_layers": 3,
      "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32, "intermediate_size": 256,
      "moe_intermediate_size": 64, "n_routed_experts": 16, "num_experts_per_tok": 4, "n_shared_experts": 1,
      "first_k_dense_replace": 1, "n_group": 4, "topk_group": 2, "routed_scaling_factor": 2.5,
      "norm_topk_prob": True, "use_qk_norm": True, "attention_bias": True, "partial_rotary_factor": 0.5,
      "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "max_position_embeddings": 4096, "tie_word_embeddings": False}


def gate_ref(logits, bias, k, n_group, topk_group, norm, scale):
    """The reference gate, one token at a time in Python."""
    T, E = logits.shape
    ws, ids = [], []
    for t in range(T):
        s = torch.sigmoid(logits[t].double())
        sel = s + bias.double()
        gsz = E // n_group
        if n_group > 1:
            gs = [sorted(sel[g * gsz:(g + 1) * gsz].tolist(), reverse=True)[:2] for g in range(n_group)]
            gsum = [sum(x) for x in gs]
            keep = sorted(range(n_group), key=lambda g: (-gsum[g], g))[:topk_group]
            sel = torch.tensor([sel[e].item() if e // gsz in keep else 0.0 for e in range(E)], dtype=torch.float64)
        order = sorted(range(E), key=lambda e: (-sel[e].item(), e))[:k]
        w = s[order]
        if norm and k > 1:
            w = w / w.sum()
        ws.append((w * scale).float())
        ids.append(order)
    return torch.stack(ws), torch.tensor(ids)


@pytest.mark.parametrize("n_group,topk_group", [(1, 1), (4, 2), (8, 3)])
def test_sigmoid_group_router_matches_reference(n_group, topk_group):
    torch.manual_seed(n_group)
    E, k = 32, 6
    lg = torch.randn(20, E) * 2
    bias = torch.randn(E) * 0.3
    w, idx = moe_ops.route_topk(lg, k, "sigmoid_group", True, bias, n_group, topk_group, 2.5)
    wr, ir = gate_ref(lg, bias, k, n_group, topk_group, True, 2.5)
    assert torch.equal(idx, ir)
    assert torch.allclose(w, wr, atol=1e-6)


def test_glm4_moe_engine_matches_dense():
    cfg = build_config(HF)
    assert cfg.router_mode == "sigmoid_group" and cfg.moe_layers == [False, True, True]
    assert cfg.shared_expert_intermediate_size == 64 and cfg.routed_scaling_factor == 2.5
    m = DecoderLM(cfg, "cpu", torch.float32).init_random(1, std=0.2)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 19, 12)]
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=7),
                                          max_model_len=128, use_cuda_graphs=False))
    out = eng.generate(prompts, max_tokens=6)
    for p, o in zip(prompts, out):
        cache = m.new_cache()
        logits = m.forward_dense(torch.tensor(p), cache)
        want = []
        for _ in range(6):
            t = int(logits[-1].argmax())
            want.append(t)
            logits = m.forward_dense(torch.tensor([t]), cache)
        assert o == want


def test_glm4_moe_checkpoint_roundtrip(tmp_path):
    from mlx_swift_lm_b200.loader.convert import save_model
    from mlx_swift_lm_b200.loader.load import load_model

    m = DecoderLM(build_config(HF), "cpu", torch.float32).init_random(4, std=0.2)
    d = str(tmp_path / "glm")
    save_model(m, d, dtype=torch.float32)
    m2, hf = load_model(d, device="cpu", dtype=torch.float32)
    assert m2.cfg.router_mode == "sigmoid_group" and m2.layers[1].router_corr is not None
    toks = torch.arange(3, 30)
    assert torch.allclose(m2.forward_dense(toks, m2.new_cache()), m.forward_dense(toks, m.new_cache()), atol=1e-4)
