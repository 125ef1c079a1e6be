"""Qwen3-VL on CPU against the transformers implementation: the vision tower
(learned position grid resampled per image, GELU-tanh blocks, merger and
deepstack mergers) and greedy generation through the paged engine from a
prompt holding an image (interleaved M-RoPE, deepstack features added after
the first decoder layers, the prompt prefilled in several chunks)."""
import json

import pytest
import torch

pytest.importorskip("transformers.models.qwen3_vl")
from safetensors.torch import save_file  # noqa: E402
from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration  # noqa: E402

from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig  # noqa: E402
from mlx_swift_lm_b200.api.media import MediaInput, process_image  # noqa: E402
from mlx_swift_lm_b200.engine.types import SamplingParams  # noqa: E402
from mlx_swift_lm_b200.loader.load import load_model  # noqa: E402
from mlx_swift_lm_b200.models.vlm import Qwen3VLModel  # noqa: E402

IMG = 290


def _export(tmp_path):
    text = dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=4,
                num_key_value_heads=2, head_dim=16, max_position_embeddings=1024, rope_theta=10000.0,
                rope_scaling={"rope_type": "default", "mrope_section": [4, 2, 2], "mrope_interleaved": True},
                tie_word_embeddings=False)
    vision = dict(depth=3, hidden_size=32, intermediate_size=64, num_heads=2, patch_size=8, temporal_patch_size=2,
                  spatial_merge_size=2, out_hidden_size=64, num_position_embeddings=16,
                  deepstack_visual_indexes=[0, 1], in_channels=3)
    hc = Qwen3VLConfig(text_config=text, vision_config=vision, image_token_id=IMG, video_token_id=291,
                       vision_start_token_id=288, vision_end_token_id=289)
    torch.manual_seed(0)
    hf = Qwen3VLForConditionalGeneration(hc).float().eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n and n.endswith("weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            else:
                p.copy_(0.15 * torch.randn_like(p))
    sd = {k: v.contiguous() for k, v in hf.state_dict().items()}
    d = tmp_path / "q3vl"
    d.mkdir()
    save_file(sd, str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    return hf, str(d)


def test_qwen3_vl_matches_transformers(tmp_path):
    hf, d = _export(tmp_path)
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    assert isinstance(m, Qwen3VLModel) and m.vision.cfg.kind == "qwen3"
    img = torch.rand(3, 40, 56)
    patches, grid = process_image(img, m.media_cfg)
    gt = torch.tensor([grid])
    with torch.no_grad():
        want = hf.model.visual(patches, grid_thw=gt)
    got, deep = m.vision.forward(patches, [grid])
    assert torch.allclose(got, want.pooler_output, atol=1e-4, rtol=1e-3), (got - want.pooler_output).abs().max()
    assert len(deep) == 2
    for a, b in zip(deep, want.deepstack_features):
        assert torch.allclose(a, b, atol=1e-4, rtol=1e-3)
    prompt = [1, 5, 288, IMG, 289, 7, 9, 11]
    toks, mm = m.prepare(prompt, MediaInput(images=[img]))
    n_img = toks.count(IMG)
    assert n_img == grid[1] * grid[2] // 4 and len(mm["deep"]) == 2
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2, prefill_chunk_size=5),
                                          max_model_len=256, use_cuda_graphs=False))
    s = eng.submit(Request(prompt_tokens=toks, max_tokens=6, mm=mm,
                           sampling=SamplingParams(temperature=0.0, top_logprobs=5)))
    eng.run_until_idle()
    evs = list(s)
    ids = torch.tensor([toks])
    ref, lps = [], []
    with torch.no_grad():
        for _ in range(6):
            tt = (ids == IMG).long()  # token types: text 0, image 1
            lg = hf(input_ids=ids, pixel_values=patches, image_grid_thw=gt, mm_token_type_ids=tt,
                    use_cache=False).logits[0, -1]
            t = int(lg.argmax())
            ref.append(t)
            lps.append(torch.log_softmax(lg.double(), -1))
            ids = torch.cat([ids, torch.tensor([[t]])], 1)
    assert [t for e in evs for t in e.tokens] == ref
    # logprobs pin the deepstack rows and the interleaved M-RoPE (greedy tokens alone may not)
    got = [lp for e in evs if e.logprobs for lp in e.logprobs]
    assert len(got) == 6
    for g, want in zip(got, lps):
        for tok, v in g.top:
            assert abs(v - float(want[tok])) < 2e-3, (tok, v, float(want[tok]))
