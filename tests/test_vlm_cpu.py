"""Qwen2-VL path on CPU: media preprocessing, M-RoPE indices, the vision
tower against a plain PyTorch re-statement, and multimodal rows through the
engine (chunk-boundary independence, decode after the image)."""
import math

import numpy as np
import torch

from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.api.media import MediaConfig, MediaInput, patchify, process_image, target_size
from mlx_swift_lm_b200.engine.types import SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.models.vision import QwenVisionTower, VisionConfig
from mlx_swift_lm_b200.models.vlm import Qwen2VLModel, get_rope_index

IMG, VID = 4000, 4001


def test_target_size_and_patchify():
    assert target_size(100, 200, 28, 56 * 56, 28 * 28 * 1280) == (112, 196)
    h, w = target_size(2000, 3000, 28, 56 * 56, 28 * 28 * 64)
    assert h % 28 == 0 and w % 28 == 0 and h * w <= 28 * 28 * 64
    cfg = MediaConfig()
    x = torch.randn(1, 3, 56, 84)
    p, g = patchify(x, cfg)
    assert g == (1, 4, 6) and p.shape == (24, 3 * 2 * 14 * 14)
    # the first 4 patches are the top-left 2x2 block (merge order), frame repeated in time
    blk = x[0, :, :14, :14].reshape(3, 1, 14, 14).expand(3, 2, 14, 14)
    assert torch.allclose(p[0], blk.reshape(-1))
    assert torch.allclose(p[1], x[0, :, :14, 14:28].reshape(3, 1, 14, 14).expand(3, 2, 14, 14).reshape(-1))


def test_rope_index():
    toks = [1, 2] + [IMG] * 4 + [3]
    pos, delta = get_rope_index(toks, [(1, 4, 4)], IMG, VID, 2)
    assert pos.tolist() == [[0, 1, 2, 2, 2, 2, 4], [0, 1, 2, 2, 3, 3, 4], [0, 1, 2, 3, 2, 3, 4]]
    assert delta == 5 - 7


def _plain_tower(t: QwenVisionTower, patches, grids):
    c = t.cfg
    E, NH, D = c.embed_dim, c.num_heads, c.head_dim
    ln = torch.nn.functional.layer_norm
    x = patches.float() @ t.patch_w.float().t()
    tab = t.rotary_table(grids)
    cos, sin = tab[:, :D // 2].repeat(1, 2), tab[:, D // 2:].repeat(1, 2)

    def rot(v):  # rotate-half
        h1, h2 = v[..., :D // 2], v[..., D // 2:]
        return v * cos[:, None] + torch.cat([-h2, h1], -1) * sin[:, None]

    lens = [h * w for tt, h, w in grids for _ in range(tt)]
    for b in t.blocks:
        h = ln(x, (E,), b.norm1_w, b.norm1_b, c.eps)
        q, k, v = (h @ b.qkv_w.t() + b.qkv_b).reshape(-1, 3, NH, D).unbind(1)
        q, k = rot(q), rot(k)
        outs, o = [], 0
        for n in lens:
            s = torch.einsum("qhd,khd->hqk", q[o:o + n], k[o:o + n]) / math.sqrt(D)
            outs.append(torch.einsum("hqk,khd->qhd", s.softmax(-1), v[o:o + n]))
            o += n
        x = x + torch.cat(outs).reshape(-1, E) @ b.proj_w.t() + b.proj_b
        h = ln(x, (E,), b.norm2_w, b.norm2_b, c.eps)
        f = h @ b.fc1_w.t() + b.fc1_b
        x = x + (f * torch.sigmoid(1.702 * f)) @ b.fc2_w.t() + b.fc2_b
    hq = ln(x, (E,), t.ln_q_w, t.ln_q_b, c.eps).reshape(-1, 4 * E)
    return torch.nn.functional.gelu(hq @ t.m1_w.t() + t.m1_b) @ t.m2_w.t() + t.m2_b


def _vcfg():
    return VisionConfig(depth=2, embed_dim=128, num_heads=2, hidden_size=256)


def test_vision_tower_matches_plain_pytorch():
    t = QwenVisionTower(_vcfg()).init_random(1, std=0.05)
    imgs = [np.random.default_rng(0).integers(0, 255, (60, 90, 3), dtype=np.uint8),
            np.random.default_rng(1).integers(0, 255, (40, 40, 3), dtype=np.uint8)]
    ps, gs = zip(*[process_image(im, MediaConfig()) for im in imgs])
    patches, grids = torch.cat(ps), list(gs)
    got = t.forward(patches, grids)
    want = _plain_tower(t, patches, grids)
    assert got.shape == (sum(a * b * c for a, b, c in grids) // 4, 256)
    assert torch.allclose(got, want, atol=1e-4)


def _vlm():
    cfg = tiny_qwen3()
    cfg.model_type = "qwen2_vl"
    cfg.rope_scaling = {"type": "mrope", "mrope_section": [8, 12, 12]}
    return Qwen2VLModel(cfg, _vcfg(), image_token_id=IMG, video_token_id=VID,
                        mrope_section=[8, 12, 12]).init_random(2, std=0.2)


def test_vlm_engine_chunking_and_decode():
    m = _vlm()
    img = np.random.default_rng(5).integers(0, 255, (56, 84, 3), dtype=np.uint8)
    toks, mm = m.prepare([5, 6, 7, IMG, 8, 9], MediaInput(images=[img]))
    assert len(toks) == 5 + 6 and mm["embeds"].shape == (6, 256)

    def run(chunk):
        eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2,
                                                                        prefill_chunk_size=chunk),
                                              max_model_len=128, use_cuda_graphs=False))
        s = eng.submit(Request(prompt_tokens=toks, max_tokens=8, sampling=SamplingParams(temperature=0.0), mm=mm))
        # a text-only request in the same batches
        t = eng.submit(Request(prompt_tokens=[11, 12, 13, 14], max_tokens=8, sampling=SamplingParams(temperature=0.0)))
        eng.run_until_idle()
        return s.tokens(), t.tokens()

    a, b = run(64), run(3)  # the image span crosses chunk boundaries at 3
    assert a == b
    # the image changes the continuation (its embeddings are used)
    img2 = np.random.default_rng(6).integers(0, 255, (56, 84, 3), dtype=np.uint8)
    toks2, mm2 = m.prepare([5, 6, 7, IMG, 8, 9], MediaInput(images=[img2]))
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=128,
                                          use_cuda_graphs=False))
    s = eng.submit(Request(prompt_tokens=toks2, max_tokens=8, sampling=SamplingParams(temperature=0.0), mm=mm2))
    eng.run_until_idle()
    x1 = m.prepare([IMG], MediaInput(images=[img]))[1]["embeds"]
    x2 = m.prepare([IMG], MediaInput(images=[img2]))[1]["embeds"]
    assert not torch.allclose(x1, x2)


def test_mrope_rows_reduce_to_rope_for_text():
    m = _vlm()
    pos = torch.arange(0, 50)
    assert torch.allclose(m._rope_rows(pos[None].expand(3, -1)), m.cos_sin[pos], atol=1e-6)


def test_vlm_checkpoint_roundtrip_and_container(tmp_path):
    from mlx_swift_lm_b200.api.container import ModelContainer
    from mlx_swift_lm_b200.api.generate import GenerateParameters
    from mlx_swift_lm_b200.loader.convert import save_model
    from mlx_swift_lm_b200.loader.load import load_model

    m = _vlm()
    d = str(tmp_path / "vl")
    save_model(m, d, dtype=torch.float32)
    m2, hf = load_model(d, device="cpu", dtype=torch.float32)
    assert isinstance(m2, Qwen2VLModel) and hf["model_type"] == "qwen2_vl"
    img = np.random.default_rng(9).integers(0, 255, (56, 56, 3), dtype=np.uint8)
    e1 = m.prepare([IMG], MediaInput(images=[img]))[1]["embeds"]
    e2 = m2.prepare([IMG], MediaInput(images=[img]))[1]["embeds"]
    assert torch.allclose(e1, e2, atol=1e-5)
    c = ModelContainer(m2, engine_config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2),
                                                      max_model_len=128, use_cuda_graphs=False))
    toks, _, info = c.generate([5, IMG, 6], params=GenerateParameters(temperature=0.0, max_tokens=5), images=[img])
    assert len(toks) == 5 and info.prompt_tokens == 2 + 4


def test_qwen25_vision_tower_matches_transformers():
    """Qwen2.5-VL tower (window attention with full-attention blocks, RMSNorm,
    biased SwiGLU of a width that is not a multiple of 64, RMSNorm merger,
    window order restored) against the transformers implementation."""
    import pytest

    tf = pytest.importorskip("transformers.models.qwen2_5_vl.modeling_qwen2_5_vl")
    from transformers.models.qwen2_5_vl.configuration_qwen2_5_vl import Qwen2_5_VLVisionConfig

    hc = Qwen2_5_VLVisionConfig(depth=4, hidden_size=64, intermediate_size=100, num_heads=2, patch_size=14,
                                spatial_merge_size=2, temporal_patch_size=2, window_size=56,
                                fullatt_block_indexes=[1, 3], out_hidden_size=96)
    torch.manual_seed(0)
    hf = tf.Qwen2_5_VisionTransformerPretrainedModel._from_config(hc).float().eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            p.copy_((1.0 + 0.1 * torch.randn_like(p)) if n.endswith("norm1.weight") or n.endswith("norm2.weight")
                    or n.endswith("ln_q.weight") else 0.1 * torch.randn_like(p))
    grids = [(1, 8, 12), (2, 4, 6)]
    N = sum(t * h * w for t, h, w in grids)
    patches = torch.randn(N, 3 * 2 * 14 * 14, generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        want = hf(patches, grid_thw=torch.tensor(grids)).pooler_output
    vc = VisionConfig.from_hf(hc.to_dict(), 96, "qwen2_5")
    assert vc.embed_dim == 64 and vc.fullatt_blocks == (1, 3) and vc.hidden_size == 96
    tower = QwenVisionTower.from_tensors(vc, {"visual." + k: v for k, v in hf.state_dict().items()}, "cpu",
                                         torch.float32)
    got = tower.forward(patches, grids)
    assert got.shape == want.shape
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-3), (got - want).abs().max()
