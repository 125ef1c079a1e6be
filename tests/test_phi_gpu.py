"""Phi-2 style model (LayerNorm with bias, parallel attention + GELU MLP,
partial rotary, biased head) through the engine on the GPU: graphs vs eager,
and the dense forward against the fp32 CPU forward."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.families import build_config

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_phi_engine_on_gpu():
    hf = {"model_type": "phi", "vocab_size": 512, "hidden_size": 256, "num_hidden_layers": 3,
          "num_attention_heads": 4, "intermediate_size": 512, "partial_rotary_factor": 0.5}
    m = DecoderLM(build_config(hf), DEV, torch.bfloat16).init_random(0, std=0.05)
    m.norm_b = torch.randn(256, device=DEV, dtype=torch.bfloat16) * 0.1
    m.lm_head_b = torch.randn(512, device=DEV) * 0.1
    for L in m.layers:
        L.ln1_b = torch.randn(256, device=DEV, dtype=torch.bfloat16) * 0.1
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=16) == eng(False).generate(ps, max_tokens=16)
    p = torch.tensor(ps[1])
    lg = m.forward_dense(p.to(DEV), m.new_cache()).float().cpu()
    mc = m.clone_to("cpu", torch.float32)
    r = mc.forward_dense(p, mc.new_cache())
    assert ((lg - r).norm() / r.norm()).item() < 0.05
