"""Qwen2-VL on the GPU: vision tower (quick-GELU epilogue, per-token 2-D
rotary table, bidirectional attention per frame) against its fp32 CPU
oracle, and multimodal requests through the engine with decode graphs."""
import numpy as np
import pytest
import torch

from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.api.media import MediaInput
from mlx_swift_lm_b200.engine.types import SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.models.vision import VisionConfig
from mlx_swift_lm_b200.models.vlm import Qwen2VLModel

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
IMG, VID = 4000, 4001


def _vlm(device, dtype):
    cfg = tiny_qwen3()
    cfg.model_type = "qwen2_vl"
    cfg.rope_scaling = {"type": "mrope", "mrope_section": [8, 12, 12]}
    v = VisionConfig(depth=2, embed_dim=128, num_heads=2, hidden_size=256)
    return Qwen2VLModel(cfg, v, "cpu", torch.float32, IMG, VID, [8, 12, 12]).init_random(2, std=0.1).clone_to(
        device, dtype)


def test_vision_tower_gpu_matches_cpu():
    mc = _vlm("cpu", torch.float32)
    mg = mc.clone_to(DEV, torch.bfloat16)
    img = np.random.default_rng(1).integers(0, 255, (112, 168, 3), dtype=np.uint8)
    ec = mc.prepare([IMG], MediaInput(images=[img]))[1]["embeds"]
    eg = mg.prepare([IMG], MediaInput(images=[img]))[1]["embeds"].float().cpu()
    cos = torch.nn.functional.cosine_similarity(ec, eg, dim=-1)
    assert (cos > 0.995).all(), cos.min()


def test_vlm_engine_graphs_match_eager():
    m = _vlm(DEV, torch.bfloat16)
    img = np.random.default_rng(2).integers(0, 255, (56, 84, 3), dtype=np.uint8)
    toks, mm = m.prepare([5, 6, IMG, 7], MediaInput(images=[img]))

    def run(graphs):
        eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2,
                                                                        prefill_chunk_size=4),
                                              max_model_len=128, use_cuda_graphs=graphs, graph_buckets=(1, 2)))
        a = eng.submit(Request(prompt_tokens=toks, max_tokens=10, sampling=SamplingParams(temperature=0.0), mm=mm))
        b = eng.submit(Request(prompt_tokens=[9, 10, 11], max_tokens=10, sampling=SamplingParams(temperature=0.0)))
        eng.run_until_idle()
        return a.tokens(), b.tokens()

    assert run(True) == run(False)
