"""Block mask-diffusion engine on CPU against a direct re-statement of the
reference's single-request loops (MLXLLM/Models/NemotronLabsDiffusion.swift
``diffusionGenerate`` / ``linearSpecGenerate``) over the dense-cache forward,
batched requests against single ones, the fused greedy-confidence op, and
the Nemotron-Labs-Diffusion checkpoint layout."""
import math

import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, ops
from mlx_swift_lm_b200.engine.block_diffusion import (BlockDiffusionEngine, DiffusionConfig, DiffusionRequest,
                                                      diffusion_generate, linear_spec_generate, transfer_schedule)
from mlx_swift_lm_b200.models.config import tiny_qwen3

MASK = 3


def _model(seed=5, std=0.3):
    c = tiny_qwen3()
    c.extra["mask_token_id"] = MASK
    c.extra["diffusion_block"] = 8
    return DecoderLM(c, "cpu", torch.float32).init_random(seed, std=std)


def _scores(lg):
    lf = lg.float()
    return lf.argmax(-1).tolist(), torch.exp(lf.max(-1).values - torch.logsumexp(lf, -1)).tolist(), \
        lf.max(-1).values.tolist()


def ref_diffusion(m, prompt, max_new, B, thr, eos):
    cache = m.new_cache()
    x = list(prompt)
    m.forward_dense(torch.tensor(prompt), cache)
    for _ in range(max_new // B):
        x += [MASK] * B
        s = len(x) - B
        sched = transfer_schedule(B, B)
        for step in range(B):
            masked = [i for i in range(B) if x[s + i] == MASK]
            if not masked:
                break
            lg = m.forward_dense(torch.tensor(x[s:s + B]), cache, bidirectional=True)
            cache.trim(B)
            tok, conf, mx = _scores(lg)
            if thr and thr > 0:
                commit = [i for i in masked if conf[i] >= thr]
                if not commit:
                    best = masked[0]
                    for i in masked:
                        if conf[i] > conf[best]:
                            best = i
                    commit = [best]
            else:
                commit = sorted(masked, key=lambda i: (-mx[i], i))[:sched[step]]
            for i in commit:
                x[s + i] = tok[i]
            if eos is not None and eos in x[s:s + B]:
                fe = x[s:s + B].index(eos)
                if MASK not in x[s:s + fe]:
                    break
        m.forward_dense(torch.tensor(x[s:s + B]), cache)
        if eos is not None and eos in x[len(prompt):]:
            return x[:len(prompt) + x[len(prompt):].index(eos) + 1]
    return x


def ref_linear_spec(m, prompt, max_new, B, thr, eos):
    cache = m.new_cache()
    lg = m.forward_dense(torch.tensor(prompt), cache)
    nxt = int(lg[-1].argmax())
    gen = [nxt]
    if eos is not None and nxt == eos:
        return prompt + gen
    total = 1
    while total < max_new:
        before = cache.offset
        block = [nxt] + [MASK] * (B - 1)
        while MASK in block:
            lg = m.forward_dense(torch.tensor(block), cache, bidirectional=True)
            cache.trim(B)
            tok, conf, _ = _scores(lg)
            if thr > 0:
                any_c, best, bc = False, -1, -math.inf
                for i in range(B):
                    if block[i] != MASK:
                        continue
                    if conf[i] >= thr:
                        block[i] = tok[i]
                        any_c = True
                    if conf[i] > bc:
                        bc, best = conf[i], i
                if not any_c and best >= 0:
                    block[best] = tok[best]
            else:
                for i in range(B):
                    if block[i] == MASK:
                        block[i] = tok[i]
                break
        lg = m.forward_dense(torch.tensor(block), cache)
        ar = lg.argmax(-1).tolist()
        acc = 0
        while acc < B - 1 and ar[acc] == block[acc + 1]:
            acc += 1
        acc += 1
        new = ar[:acc]
        gen += new
        total += acc
        cache.trim(cache.offset - (before + acc))
        nxt = new[-1]
        if eos is not None and eos in new:
            gen = gen[:len(gen) - len(new)] + new[:new.index(eos) + 1]
            break
    return prompt + gen[:max_new]


def test_transfer_schedule():
    assert transfer_schedule(10, 4) == [3, 3, 2, 2]
    assert transfer_schedule(8, 8) == [1] * 8


@pytest.mark.parametrize("thr", [0.9, 0.02, None])
def test_diffusion_matches_reference_loop(thr):
    m = _model()
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(4, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 13, 9)]
    eng = BlockDiffusionEngine(m, DiffusionConfig(max_rows=4, prefill_chunk=6, kv_tokens=1024))
    free0 = eng.kv.free_pages
    reqs = [DiffusionRequest(p, 16, 8, thr) for p in prompts]
    out = eng.generate(reqs)
    for p, (toks, nfe) in zip(prompts, out):
        assert toks == ref_diffusion(m, p, 16, 8, thr, None)
        assert MASK not in toks[len(p):]
        assert nfe >= 3
    # batched == one at a time
    for p, (toks, _) in zip(prompts, out):
        assert diffusion_generate(m, p, 16, 8, thr)[0] == toks
    assert not eng.rows and eng.kv.free_pages == free0  # every page returned


def test_diffusion_stops_at_eos():
    m = _model()
    p = list(range(10, 20))
    free = diffusion_generate(m, p, 24, 8, 0.02)[0]
    eos = free[len(p) + 5]  # a token the model does produce
    toks, _ = diffusion_generate(m, p, 24, 8, 0.02, eos_token_id=eos)
    assert toks == ref_diffusion(m, p, 24, 8, 0.02, eos)
    assert toks[-1] == eos and eos not in toks[len(p):-1]


@pytest.mark.parametrize("thr", [0.0, 0.05])
def test_linear_spec_matches_reference_loop(thr):
    m = _model(seed=7)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(4, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 11)]
    eng = BlockDiffusionEngine(m, DiffusionConfig(max_rows=4, kv_tokens=1024))
    reqs = [DiffusionRequest(p, 20, 4, thr, mode="linear_spec") for p in prompts]
    for p, (toks, _) in zip(prompts, eng.generate(reqs)):
        assert toks == ref_linear_spec(m, p, 20, 4, thr, None)
        assert linear_spec_generate(m, p, 20, 4, thr)[0] == toks
    # the verifier accepts only greedy-consistent tokens: the output equals plain greedy decoding
    p = prompts[0]
    cache = m.new_cache()
    lg = m.forward_dense(torch.tensor(p), cache)
    greedy = []
    for _ in range(20):
        t = int(lg[-1].argmax())
        greedy.append(t)
        lg = m.forward_dense(torch.tensor([t]), cache)
    assert linear_spec_generate(m, p, 20, 4, thr)[0][len(p):] == greedy


def test_argmax_confidence_reference():
    x = torch.randn(5, 77)
    x[2, 10] = 50.0
    tok, conf, mx = ops.argmax_confidence(x)
    assert tok.tolist() == x.argmax(-1).tolist()
    assert torch.allclose(conf, torch.softmax(x, -1).max(-1).values, atol=1e-6)
    assert conf[2] > 0.999 and torch.equal(mx, x.max(-1).values)


def test_rejects_bad_requests():
    m = _model()
    eng = BlockDiffusionEngine(m, DiffusionConfig(kv_tokens=256))
    with pytest.raises(ValueError):
        eng.submit(DiffusionRequest([5, 6], 10, 8))
    with pytest.raises(ValueError):
        eng.submit(DiffusionRequest([], 8, 8))


def test_nemotron_labs_diffusion_checkpoint(tmp_path):
    from mlx_swift_lm_b200.loader.convert import export_tensors, write_shards
    from mlx_swift_lm_b200.loader.load import load_model
    import json

    c = tiny_qwen3()
    c.qk_norm = False
    m = DecoderLM(c, "cpu", torch.float32).init_random(2, std=0.2)
    t = export_tensors(m)
    t = {("encoder." + k[len("model."):] if k.startswith("model.") else k): v for k, v in t.items()}
    t["diffusion_head.weight"] = t.pop("lm_head.weight", t["encoder.embed_tokens.weight"].clone())
    t["encoder.layers.0.self_attn.rotary_emb.inv_freq"] = torch.ones(4)
    d = tmp_path / "nld"
    d.mkdir()
    hf = {"model_type": "nemotron_labs_diffusion", "hidden_size": c.hidden_size, "num_hidden_layers": c.num_layers,
          "intermediate_size": c.intermediate_size, "num_attention_heads": c.num_heads,
          "num_key_value_heads": c.num_kv_heads, "head_dim": c.head_dim, "rms_norm_eps": c.rms_norm_eps,
          "vocab_size": c.vocab_size, "mask_token_id": 7, "block_size": 16, "tie_word_embeddings": False,
          "rope_parameters": {"rope_theta": 500000.0, "rope_type": "default", "llama_4_scaling_beta": 0.1,
                              "original_max_position_embeddings": 16}}
    (d / "config.json").write_text(json.dumps(hf))
    write_shards(t, str(d))
    lm, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert lm.cfg.extra["mask_token_id"] == 7 and lm.cfg.extra["diffusion_block"] == 16
    assert lm.cfg.rope_theta == 500000.0 and lm.cfg.extra["attn_pos_scale"] == (0.1, 16)
    assert torch.equal(lm.lm_head, t["diffusion_head.weight"])
    eng = BlockDiffusionEngine(lm, DiffusionConfig(kv_tokens=512))
    assert eng.mask == 7 and eng.default_block == 16
    # positions past original_max scale the queries: paged and dense paths agree
    p = list(range(20, 45))
    toks, _ = eng.generate([DiffusionRequest(p, 16, None, 0.5)])[0]
    assert toks == diffusion_ref_for(lm, p)


def diffusion_ref_for(lm, p):
    global MASK
    old, MASK = MASK, 7
    try:
        return ref_diffusion(lm, p, 16, 16, 0.5, None)
    finally:
        MASK = old
