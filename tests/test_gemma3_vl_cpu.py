"""Gemma 3 vision-language model on CPU against the transformers
implementation: the SigLIP tower and pooled projector, and greedy
generation through the paged engine from a prompt that holds an image."""
import json

import pytest
import torch

pytest.importorskip("transformers.models.gemma3")
from safetensors.torch import save_file  # noqa: E402
from transformers import Gemma3Config, Gemma3ForConditionalGeneration  # noqa: E402

from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig  # noqa: E402
from mlx_swift_lm_b200.api.media import MediaInput  # noqa: E402
from mlx_swift_lm_b200.engine.types import SamplingParams  # noqa: E402
from mlx_swift_lm_b200.loader.load import load_model  # noqa: E402
from mlx_swift_lm_b200.models.siglip import siglip_pixels  # noqa: E402

IMG = 299


def _export(tmp_path):
    text = dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2,
                num_key_value_heads=1, head_dim=32, sliding_window=16, query_pre_attn_scalar=32,
                rope_theta=10000.0, rope_local_base_freq=10000.0, max_position_embeddings=512)
    vision = dict(hidden_size=48, intermediate_size=96, num_hidden_layers=2, num_attention_heads=2,
                  image_size=56, patch_size=14, num_channels=3)
    hc = Gemma3Config(text_config=text, vision_config=vision, mm_tokens_per_image=4, image_token_index=IMG,
                      boi_token_index=297, eoi_token_index=298)
    torch.manual_seed(0)
    hf = Gemma3ForConditionalGeneration(hc).float().eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n and n.endswith("weight"):
                p.copy_(0.1 * torch.randn_like(p) + (1.0 if "layer_norm" in n or "post_layernorm" in n else 0.0))
            elif "mm_input_projection" in n:
                p.copy_(0.2 * torch.randn_like(p))
            else:
                p.copy_(0.15 * torch.randn_like(p))
    sd = {k: v.contiguous() for k, v in hf.state_dict().items() if k != "lm_head.weight"}
    d = tmp_path / "g3vl"
    d.mkdir()
    save_file(sd, str(d / "model.safetensors"))
    cfg = hc.to_dict()
    (d / "config.json").write_text(json.dumps(cfg))
    return hf, str(d)


def test_gemma3_vl_matches_transformers(tmp_path):
    hf, d = _export(tmp_path)
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    img = torch.rand(3, 70, 90)
    pix = siglip_pixels(img, 56)
    with torch.no_grad():
        want = hf.model.get_image_features(pixel_values=pix[None]).pooler_output.reshape(-1, 64)
    got = m.image_embeddings(pix[None])
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-3), (got - want).abs().max()
    prompt = [2, 5, 297, IMG, 298, 7, 9]
    toks, mm = m.prepare(prompt, MediaInput(images=[img]))
    assert toks.count(IMG) == 4 and mm["embeds"].shape == (4, 64)
    eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2, prefill_chunk_size=5),
                                          max_model_len=128, use_cuda_graphs=False))
    s = eng.submit(Request(prompt_tokens=toks, max_tokens=6, sampling=SamplingParams(temperature=0.0), mm=mm))
    eng.run_until_idle()
    got_toks = s.tokens()
    ids = torch.tensor([toks])
    ref = []
    with torch.no_grad():
        for _ in range(6):
            lg = hf(input_ids=ids, pixel_values=pix[None]).logits[0, -1]
            t = int(lg.argmax())
            ref.append(t)
            ids = torch.cat([ids, torch.tensor([[t]])], 1)
    assert got_toks == ref
