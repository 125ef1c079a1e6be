"""Gemma 4 through the engine on the GPU (sliding layers at head dim 256,
global layers at 512 on the wide decode kernel, KV-shared layers, per-layer
inputs; and the MoE variant with k_eq_v): CUDA graphs vs eager, and the GPU
dense forward against the fp32 CPU forward."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.families import build_config
from mlx_swift_lm_b200.ops import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

LT = ["sliding_attention", "sliding_attention", "full_attention", "sliding_attention", "sliding_attention",
      "full_attention"]
ROPE = {"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
        "full_attention": {"rope_type": "proportional", "partial_rotary_factor": 0.25, "rope_theta": 1000000.0}}


def _hf(**kw):
    d = dict(model_type="gemma4_text", vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=6,
             num_attention_heads=4, num_key_value_heads=1, head_dim=256, global_head_dim=512, sliding_window=32,
             layer_types=LT, num_kv_shared_layers=2, hidden_size_per_layer_input=64, vocab_size_per_layer_input=512,
             use_double_wide_mlp=True, final_logit_softcapping=30.0, rope_parameters=ROPE, rms_norm_eps=1e-6,
             max_position_embeddings=4096)
    d.update(kw)
    return d


@pytest.mark.parametrize("variant", ["e2b_like", "k_eq_v", "moe_k_eq_v"])
def test_gemma4_engine_on_gpu(variant):
    kw = {}
    if variant != "e2b_like":
        kw = dict(hidden_size_per_layer_input=0, num_kv_shared_layers=0, use_double_wide_mlp=False,
                  attention_k_eq_v=True, num_global_key_value_heads=2)
    if variant == "moe_k_eq_v":
        kw.update(enable_moe_block=True, num_experts=8, top_k_experts=2, moe_intermediate_size=128)
    hf = _hf(**kw)
    m = DecoderLM(build_config(hf), DEV, torch.bfloat16).init_random(0, std=0.05)
    # attention scale is 1: unit q/k norm weights make random-init scores ~N(0, D) and the
    # softmax an argmax that bf16 rounding flips; D^-1/4 on each keeps them O(1)
    for li, L in enumerate(m.layers):
        d = m.geom(li)[1]
        L.q_norm.mul_(d ** -0.25)
        if L.k_norm is not None:
            L.k_norm.mul_(d ** -0.25)
        if L.router is not None:  # decisive top-k margins: bf16 vs fp32 must pick the same experts
            L.router.mul_(8.0)
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=12) == eng(False).generate(ps, max_tokens=12)
    assert _lib.read_status().get("attn_wide", 0) == 0
    p = torch.tensor(ps[2])
    lg = m.forward_dense(p.to(DEV), m.new_cache()).float().cpu()
    mc = m.clone_to("cpu", torch.float32)
    r = mc.forward_dense(p, mc.new_cache())
    if variant != "moe_k_eq_v":
        assert ((lg - r).norm() / r.norm()).item() < 0.05
    else:
        # bf16 rounding flips the top-2 choice of a few tokens after a few
        # layers (the fp32 vs bf16 CPU forwards differ the same way); the
        # typical token must still match closely
        tok = ((lg - r).norm(dim=-1) / r.norm(dim=-1))
        assert tok.median().item() < 0.05 and (tok < 0.05).float().mean().item() > 0.6


def test_gemma4_moe_block_and_router_on_gpu():
    """The MoE feed-forward of one layer (router on the normed residual with
    per-expert scales, GeGLU experts, the dense branch and the four norms) on
    the GPU against the fp32 CPU restatement of the same weights."""
    hf = _hf(hidden_size_per_layer_input=0, num_kv_shared_layers=0, use_double_wide_mlp=False,
             enable_moe_block=True, num_experts=8, top_k_experts=2, moe_intermediate_size=128)
    m = DecoderLM(build_config(hf), DEV, torch.bfloat16).init_random(3, std=0.05)
    L = m.layers[0]
    L.router.mul_(8.0)
    mc = m.clone_to("cpu", torch.float32)
    x = (torch.randn(37, 256, generator=torch.Generator().manual_seed(5)) * 0.5).to(torch.bfloat16)
    w, idx = m._route(L, x.to(DEV))
    wc, ic = mc._route(mc.layers[0], x.float())
    assert torch.equal(idx.long().cpu().sort(-1).values, ic.long().sort(-1).values)
    y = m._ffn(L, x.to(DEV)).float().cpu()
    yc = mc._ffn(mc.layers[0], x.float())
    assert ((y - yc).norm() / yc.norm()).item() < 0.03
