"""DeepSeek-V3-style model (multi-head latent attention with zero-padded
heads in the paged cache, sigmoid group router, shared experts) through the
engine on the GPU: CUDA graphs vs eager, and the GPU dense forward against
the fp32 CPU forward."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.families import build_config

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

HF = dict(model_type="deepseek_v3", vocab_size=512, hidden_size=256, num_hidden_layers=3, num_attention_heads=4,
          intermediate_size=512, moe_intermediate_size=128, n_routed_experts=16, num_experts_per_tok=4,
          n_shared_experts=1, first_k_dense_replace=1, n_group=4, topk_group=2, routed_scaling_factor=2.0,
          norm_topk_prob=True, q_lora_rank=64, kv_lora_rank=128, qk_nope_head_dim=64, qk_rope_head_dim=32,
          v_head_dim=64, rms_norm_eps=1e-6, rope_theta=10000.0, max_position_embeddings=4096,
          rope_scaling={"type": "yarn", "factor": 4.0, "original_max_position_embeddings": 1024, "beta_fast": 32,
                        "beta_slow": 1, "mscale": 1.0, "mscale_all_dim": 1.0})


def test_deepseek_v3_engine_on_gpu():
    cfg = build_config(HF)
    assert cfg.head_dim == 128
    m = DecoderLM(cfg, DEV, torch.bfloat16).init_random(0, std=0.05)
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=12) == eng(False).generate(ps, max_tokens=12)
    p = torch.tensor(ps[2])
    lg = m.forward_dense(p.to(DEV), m.new_cache()).float().cpu()
    mc = m.clone_to("cpu", torch.float32)
    r = mc.forward_dense(p, mc.new_cache())
    assert ((lg - r).norm() / r.norm()).item() < 0.05
