"""PaliGemma, Idefics3 and SmolVLM (SigLIP-tower VLMs) on CPU against the
transformers implementations: connector outputs, and greedy generation
through the paged engine from a prompt that holds an image (PaliGemma's
prompt attends both ways; SmolVLM's large image is split into tiles with
row / column marker tokens)."""
import json

import pytest
import torch

pytest.importorskip("transformers.models.idefics3")
from safetensors.torch import save_file  # noqa: E402

from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig  # noqa: E402
from mlx_swift_lm_b200.api.media import MediaInput  # noqa: E402
from mlx_swift_lm_b200.engine.types import SamplingParams  # noqa: E402
from mlx_swift_lm_b200.loader.load import load_model  # noqa: E402
from mlx_swift_lm_b200.models.siglip import SiglipVLM, smolvlm_tiles  # noqa: E402

VISION = dict(hidden_size=48, intermediate_size=96, num_hidden_layers=2, num_attention_heads=2, image_size=56,
              patch_size=14, num_channels=3)
LLAMA = dict(model_type="llama", vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
             num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=512,
             rope_theta=10000.0, rms_norm_eps=1e-6, tie_word_embeddings=False)


def _randomise(hf):
    torch.manual_seed(1)
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n and n.endswith("weight"):
                base = 0.0 if ("language_model" in n and "gemma" in type(hf).__name__.lower()) else 1.0
                p.copy_(0.1 * torch.randn_like(p) + base)
            else:
                p.copy_(0.15 * torch.randn_like(p))


def _save(hf, hc, tmp_path, name, pre=None):
    sd = {k: v.contiguous() for k, v in hf.state_dict().items()}
    if sd.get("lm_head.weight") is not None and any(
            k.endswith("embed_tokens.weight") and v.data_ptr() == sd["lm_head.weight"].data_ptr() for k, v in sd.items()
            if k != "lm_head.weight"):
        del sd["lm_head.weight"]  # tied
    d = tmp_path / name
    d.mkdir()
    save_file(sd, str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    if pre is not None:
        (d / "preprocessor_config.json").write_text(json.dumps(pre))
    return str(d)


def _engine(m, chunk=64):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2,
                                                                     prefill_chunk_size=chunk),
                                           max_model_len=256, use_cuda_graphs=False))


def _greedy_ref(hf, toks, n, lps=None, **kw):
    ids = torch.tensor([toks])
    out = []
    with torch.no_grad():
        for _ in range(n):
            extra = {}
            if "token_type_ids" in kw:  # prompt = prefix (0), generated = suffix (1)
                extra["token_type_ids"] = torch.cat(
                    [torch.zeros(1, len(toks), dtype=torch.long), torch.ones(1, ids.shape[1] - len(toks),
                                                                           dtype=torch.long)], 1)
            lg = hf(input_ids=ids, use_cache=False, **{k: v for k, v in kw.items() if k != "token_type_ids"},
                    **extra).logits[0, -1]
            t = int(lg.argmax())
            out.append(t)
            if lps is not None:
                lps.append(torch.log_softmax(lg.double(), -1))
            ids = torch.cat([ids, torch.tensor([[t]])], 1)
    return out


def test_paligemma_prefix_lm_matches_transformers(tmp_path):
    from transformers import PaliGemmaConfig, PaliGemmaForConditionalGeneration

    text = dict(model_type="gemma", vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                num_attention_heads=2, num_key_value_heads=1, head_dim=32, max_position_embeddings=512)
    hc = PaliGemmaConfig(text_config=text, vision_config={**VISION, "projection_dim": 64}, image_token_index=299,
                         projection_dim=64, hidden_size=64)
    hf = PaliGemmaForConditionalGeneration(hc).float().eval()
    _randomise(hf)
    d = _save(hf, hc, tmp_path, "pali")
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    assert isinstance(m, SiglipVLM) and m.kind == "paligemma" and m.mm_tokens == 16
    img = torch.rand(3, 60, 80)
    pix = m._pixels(img)
    prompt = [2, 11, 12, 13, 108]
    toks, mm = m.prepare(prompt, MediaInput(images=[img]))
    assert toks[:16] == [299] * 16 and toks[16:] == prompt and mm["prefix_lm"]
    eng = _engine(m)
    s = eng.submit(Request(prompt_tokens=toks, max_tokens=5, mm=mm,
                           sampling=SamplingParams(temperature=0.0, top_logprobs=5)))
    eng.run_until_idle()
    lps = []
    ref = _greedy_ref(hf, toks, 5, lps, pixel_values=pix[None], token_type_ids=True)
    evs = list(s)
    assert [t for e in evs for t in e.tokens] == ref
    # logprobs pin the attention pattern (a causal prompt changes them by far more)
    got = [lp for e in evs if e.logprobs for lp in e.logprobs]
    assert len(got) == 5
    for g, want in zip(got, lps):
        for tok, v in g.top:
            assert abs(v - float(want[tok])) < 2e-3, (tok, v, float(want[tok]))
    # a prefix-LM prompt longer than one chunk is refused, not silently made causal
    with pytest.raises(ValueError):
        _engine(m, chunk=8).submit(Request(prompt_tokens=toks, max_tokens=2, mm=mm))


def test_idefics3_matches_transformers(tmp_path):
    from transformers import Idefics3Config, Idefics3ForConditionalGeneration

    hc = Idefics3Config(text_config=LLAMA, vision_config=VISION, scale_factor=2, image_token_id=290)
    hf = Idefics3ForConditionalGeneration(hc).float().eval()
    _randomise(hf)
    d = _save(hf, hc, tmp_path, "idefics3")
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    assert m.kind == "idefics3" and m.mm_tokens == 4
    img = torch.rand(3, 50, 64)
    pix = m._pixels(img)
    with torch.no_grad():
        want = hf.model.get_image_features(pixel_values=pix[None, None])
        want = getattr(want, "pooler_output", want).reshape(-1, 64)
    got = m.image_embeddings(pix[None])
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-3), (got - want).abs().max()
    prompt = [1, 20, 290, 21, 22]
    toks, mm = m.prepare(prompt, MediaInput(images=[img]))
    assert toks == [1, 20] + [290] * 4 + [21, 22]
    eng = _engine(m, chunk=3)  # image rows split across prefill chunks
    s = eng.submit(Request(prompt_tokens=toks, max_tokens=6, sampling=SamplingParams(temperature=0.0), mm=mm))
    eng.run_until_idle()
    assert s.tokens() == _greedy_ref(hf, toks, 6, pixel_values=pix[None, None])
    # no placeholder: the image tokens go to the middle of the prompt
    toks2, _ = m.prepare([1, 20, 21, 22], MediaInput(images=[img]))
    assert toks2 == [1, 20] + [290] * 4 + [21, 22]


def test_smolvlm_tiles_match_transformers(tmp_path):
    from transformers import SmolVLMConfig, SmolVLMForConditionalGeneration

    hc = SmolVLMConfig(text_config=LLAMA, vision_config=VISION, scale_factor=2, image_token_id=290)
    hf = SmolVLMForConditionalGeneration(hc).float().eval()
    _randomise(hf)
    d = _save(hf, hc, tmp_path, "smolvlm", pre={"image_mean": [0.5] * 3, "image_std": [0.5] * 3,
                                                   "do_image_splitting": True, "size": {"longest_edge": 112}})
    m, _ = load_model(d, device="cpu", dtype=torch.float32)
    assert m.tile_longest_edge == 112
    m.marker_ids = {"fake": 280, "global": [281], "newline": [10],
                    "row": lambda r, c: [200 + 10 * r + c]}
    img = torch.rand(3, 90, 120)  # -> 112 x 112 canvas of 2 x 2 tiles of 56, plus the global tile
    tiles, rows, cols = smolvlm_tiles(img, 56, 112)
    assert (rows, cols, len(tiles)) == (2, 2, 5)
    prompt = [1, 290, 21]
    toks, mm = m.prepare(prompt, MediaInput(images=[img]))
    run = []
    for r in range(2):
        for c in range(2):
            run += [280, 200 + 10 * r + c] + [290] * 4
        run += [10]
    run += [10, 280, 281] + [290] * 4 + [280]
    assert toks == [1] + run + [21] and mm["embeds"].shape == (20, 64)
    pix = torch.stack([(t - 0.5) / 0.5 for t in tiles])
    eng = _engine(m, chunk=16)
    s = eng.submit(Request(prompt_tokens=toks, max_tokens=5, sampling=SamplingParams(temperature=0.0), mm=mm))
    eng.run_until_idle()
    assert s.tokens() == _greedy_ref(hf, toks, 5, pixel_values=pix[None])
