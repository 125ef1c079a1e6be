"""Qwen2.5-VL window-attention tower and the Gemma 3 SigLIP tower on the GPU
against their fp32 CPU forwards (the SigLIP case uses head dim 72, zero-padded
to the prefill kernel's 128), and a Gemma 3 VLM request through the engine
with CUDA graphs against eager."""
import pytest
import torch

from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.api.media import MediaInput
from mlx_swift_lm_b200.engine.types import SamplingParams
from mlx_swift_lm_b200.models.families import build_config
from mlx_swift_lm_b200.models.siglip import Gemma3VLModel, SiglipConfig, SiglipVisionTower
from mlx_swift_lm_b200.models.vision import QwenVisionTower, VisionConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_qwen25_tower_gpu():
    vc = VisionConfig(depth=4, embed_dim=256, num_heads=2, hidden_size=512, kind="qwen2_5", intermediate_size=300,
                      window_size=56, fullatt_blocks=(1, 3))
    cpu = QwenVisionTower(vc).init_random(0, std=0.05)
    gpu = QwenVisionTower(vc, DEV, torch.bfloat16).init_random(0, std=0.05)
    for n, t in cpu.tensors():  # same weights on both
        if t is not None:
            if n.startswith("blocks."):
                _, i, s = n.split(".")
                setattr(gpu.blocks[int(i)], s, t.to(DEV, torch.bfloat16).contiguous())
            else:
                setattr(gpu, n, t.to(DEV, torch.bfloat16).contiguous())
    grids = [(1, 8, 12), (2, 4, 6)]
    N = sum(t * h * w for t, h, w in grids)
    x = torch.randn(N, vc.patch_dim, generator=torch.Generator().manual_seed(1))
    assert _rel(gpu.forward(x, grids).cpu(), cpu.forward(x, grids)) < 0.03


@pytest.mark.parametrize("hidden,heads", [(256, 2), (144, 2)])
def test_siglip_tower_gpu(hidden, heads):
    sc = SiglipConfig(hidden_size=hidden, intermediate_size=2 * hidden, num_layers=3, num_heads=heads,
                      image_size=112, patch_size=14)
    cpu = SiglipVisionTower(sc).init_random(0, std=0.05)
    gpu = SiglipVisionTower(sc, DEV, torch.bfloat16)
    gpu.patch_w, gpu.patch_b, gpu.pos, gpu.post_w, gpu.post_b = cpu.patch_w, cpu.patch_b, cpu.pos, cpu.post_w, \
        cpu.post_b
    gpu.layers = [{k: v for k, v in L.items() if k not in ("qkv_w", "qkv_b")} for L in cpu.layers]
    gpu.to(DEV, torch.bfloat16)
    pix = torch.randn(2, 3, 112, 112, generator=torch.Generator().manual_seed(2))
    assert _rel(gpu.forward(pix).cpu(), cpu.forward(pix)) < 0.03


def test_gemma3_vl_engine_gpu():
    hf = dict(model_type="gemma3_text", vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
              num_attention_heads=2, num_key_value_heads=1, head_dim=128, sliding_window=32, query_pre_attn_scalar=128,
              rope_theta=10000.0, rope_local_base_freq=10000.0, max_position_embeddings=1024)
    sc = SiglipConfig(hidden_size=256, intermediate_size=512, num_layers=2, num_heads=2, image_size=112,
                      patch_size=14)
    m = Gemma3VLModel(build_config(hf), sc, DEV, torch.bfloat16, image_token_id=511, mm_tokens=16)
    m.init_random(0, std=0.05)
    img = torch.rand(3, 90, 120)
    toks, mm = m.prepare([3, 5, 511, 7, 9], MediaInput(images=[img]))

    def run(graphs):
        e = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=256,
                                            use_cuda_graphs=graphs, graph_buckets=(1, 2)))
        s = e.submit(Request(prompt_tokens=toks, max_tokens=10, sampling=SamplingParams(temperature=0.0), mm=mm))
        e.run_until_idle()
        return s.tokens()

    assert run(True) == run(False)
