"""Gemma 4 text models on CPU against the transformers implementation of
the same architecture (an independent restatement used as the oracle):
per-kind head dims and KV heads, proportional partial RoPE on full layers,
KV-shared trailing layers with double-wide MLPs, per-layer inputs, k_eq_v,
the MoE block with its router, soft-capped logits; then the paged engine
against the dense forward and the KV-slab geometry."""
import json

import pytest
import torch

pytest.importorskip("transformers.models.gemma4")
from safetensors.torch import save_file  # noqa: E402
from transformers import Gemma4ForCausalLM, Gemma4TextConfig  # noqa: E402

from mlx_swift_lm_b200 import EngineConfig, EngineV2, SchedulerConfig  # noqa: E402
from mlx_swift_lm_b200.loader.load import load_model  # noqa: E402

LT = ["sliding_attention", "sliding_attention", "full_attention", "sliding_attention", "sliding_attention",
      "full_attention"]
ROPE = {"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
        "full_attention": {"rope_type": "proportional", "partial_rotary_factor": 0.25, "rope_theta": 1000000.0}}


def _hf_config(**kw):
    d = dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=6, num_attention_heads=2,
             num_key_value_heads=1, head_dim=32, global_head_dim=64, sliding_window=8, layer_types=LT,
             num_kv_shared_layers=2, hidden_size_per_layer_input=16, vocab_size_per_layer_input=300,
             use_double_wide_mlp=True, final_logit_softcapping=30.0, rope_parameters=ROPE)
    d.update(kw)
    return Gemma4TextConfig(**d)


def _export(hc, tmp_path, seed=0):
    torch.manual_seed(seed)
    hf = Gemma4ForCausalLM(hc).float().eval()
    with torch.no_grad():  # every parameter random, norms near 1
        for n, p in hf.named_parameters():
            if "norm" in n or n.endswith("scale") or n.endswith("per_expert_scale"):
                p.copy_(1.0 + 0.2 * torch.randn_like(p))
            else:
                p.copy_(0.15 * torch.randn_like(p))
        for i, layer in enumerate(hf.model.layers):
            layer.layer_scalar.fill_(0.7 + 0.1 * i)
    sd = {k: v.contiguous() for k, v in hf.state_dict().items() if k != "lm_head.weight"}
    d = tmp_path / "g4"
    d.mkdir()
    save_file(sd, str(d / "model.safetensors"))
    cfg = hc.to_dict()
    cfg["model_type"] = "gemma4_text"
    (d / "config.json").write_text(json.dumps(cfg))
    return hf, str(d)


def _hf_logits(hf, toks):
    with torch.no_grad():
        return hf(torch.tensor([toks])).logits[0].float()


@pytest.mark.parametrize("variant", ["ple_shared", "k_eq_v_moe"])
def test_gemma4_matches_transformers(tmp_path, variant):
    if variant == "ple_shared":
        hc = _hf_config()
    else:
        hc = _hf_config(hidden_size_per_layer_input=0, num_kv_shared_layers=0, use_double_wide_mlp=False,
                        attention_k_eq_v=True, num_global_key_value_heads=2, enable_moe_block=True, num_experts=8,
                        top_k_experts=2, moe_intermediate_size=64)
    hf, d = _export(hc, tmp_path)
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    toks = torch.randint(0, 300, (21,), generator=torch.Generator().manual_seed(3)).tolist()
    want = _hf_logits(hf, toks)
    got = m.forward_dense(torch.tensor(toks), m.new_cache())
    assert torch.allclose(got, want, atol=2e-3, rtol=1e-3), (got - want).abs().max()
    # incremental dense decode equals the one-shot forward
    cache = m.new_cache()
    m.forward_dense(torch.tensor(toks[:15]), cache)
    step = m.forward_dense(torch.tensor(toks[15:16]), cache)
    assert torch.allclose(step[0], want[15], atol=2e-3, rtol=1e-3)


def test_gemma4_kv_geometry_and_engine(tmp_path):
    hc = _hf_config()
    hf, d = _export(hc, tmp_path, seed=1)
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    # four layers own K/V (two shared); sliding: 1 KV head x 32, full: 1 x 64
    assert m.kv_layer_geom() == [(1, 32, 8), (1, 32, 8), (1, 64, 0), (1, 32, 8)]
    assert m.kv_index == [0, 1, 2, 3, 3, 2]
    assert m.kv_bytes_per_token(torch.float32) == 2 * 4 * (3 * 32 + 64)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=3, prefill_chunk_size=7),
                                          max_model_len=96, use_cuda_graphs=False))
    assert [tuple(s) for s in eng.kv.group_shapes] == [(1, 32), (1, 64)]
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 300, (n,), generator=g).tolist() for n in (5, 30, 17)]
    out = eng.generate(prompts, max_tokens=6)
    for p, o in zip(prompts, out):
        want = []
        toks = list(p)
        for _ in range(6):
            t = int(_hf_logits(hf, toks)[-1].argmax())
            want.append(t)
            toks.append(t)
        assert o == want
