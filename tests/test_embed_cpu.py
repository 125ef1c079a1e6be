"""Encoders (BERT / DistilBERT-style / NomicBERT-style) against a plain
PyTorch re-statement, pooling strategies, cross-encoder and decoder
rerankers, decoder last-token embeddings (CPU, fp32)."""
import math

import torch

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.api.embed import Embedder, Pooling, RerankScore, Reranker
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.models.encoder import EncoderConfig, EncoderModel
from mlx_swift_lm_b200.ops import reference as ref


def _plain_bert(m: EncoderModel, ids: list[int]) -> torch.Tensor:
    """Single-sequence post-norm encoder in plain PyTorch (no packing, no pages)."""
    cfg = m.cfg
    n = len(ids)
    x = m.word[torch.tensor(ids)].float()
    if m.pos is not None:
        x = x + m.pos[torch.arange(n) + cfg.position_offset].float()
    if m.type is not None:
        x = x + m.type[0].float()
    ln = torch.nn.functional.layer_norm
    H, NH = cfg.hidden_size, cfg.num_heads
    D = H // NH
    x = ln(x, (H,), m.emb_ln_w, m.emb_ln_b, cfg.layer_norm_eps)
    pos = torch.arange(n, dtype=torch.int32)
    for L in m.layers:
        qkv = x @ L.wqkv.t() + (L.bqkv if L.bqkv is not None else 0)
        q, k, v = qkv.split(H, -1)
        q, k, v = (t.reshape(n, NH, D) for t in (q, k, v))
        if cfg.rotary:
            q = ref.apply_rope_ref(q, pos, m.cos_sin, m.rot_dim)
            k = ref.apply_rope_ref(k, pos, m.cos_sin, m.rot_dim)
        att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(D), -1)
        a = torch.einsum("hqk,khd->qhd", att, v).reshape(n, H)
        x = ln(x + a @ L.wo.t() + (L.bo if L.bo is not None else 0), (H,), L.ln1_w, L.ln1_b, cfg.layer_norm_eps)
        if cfg.hidden_act == "swiglu":
            h = ref.gemm_ref(x, L.w1, "swiglu", bias=L.b1)
        else:
            h = torch.nn.functional.gelu(x @ L.w1.t() + (L.b1 if L.b1 is not None else 0))
        x = ln(x + h @ L.w2.t() + (L.b2 if L.b2 is not None else 0), (H,), L.ln2_w, L.ln2_b, cfg.layer_norm_eps)
    return x


def _cfg(**kw):
    c = EncoderConfig(vocab_size=300, hidden_size=128, num_layers=2, num_heads=2, intermediate_size=256,
                      max_position_embeddings=64)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_encoder_matches_plain_pytorch():
    for kw in ({}, {"position_offset": 2, "type_vocab_size": 1}, {"rotary": True, "hidden_act": "swiglu",
                                                                   "bias": False}):
        m = EncoderModel(_cfg(**kw)).init_random(1, std=0.1)
        seqs = [list(range(5, 22)), list(range(40, 47)), list(range(100, 133))]
        x, cu = m.forward(seqs)
        for r, s in enumerate(seqs):
            want = _plain_bert(m, s)
            assert torch.allclose(x[cu[r]:cu[r + 1]], want, atol=2e-4), kw


def test_pooling_strategies():
    x = torch.arange(24, dtype=torch.float32).reshape(6, 4)
    cu = [0, 2, 6]
    assert torch.equal(Pooling("first")(x, cu), x[[0, 2]])
    assert torch.equal(Pooling("last")(x, cu), x[[1, 5]])
    assert torch.allclose(Pooling("mean")(x, cu), torch.stack([x[:2].mean(0), x[2:].mean(0)]))
    assert torch.equal(Pooling("max")(x, cu), x[[1, 5]])
    e = Pooling("mean", dimension=3)(x, cu, normalize=True)
    assert e.shape == (2, 3) and torch.allclose(e.norm(dim=-1), torch.ones(2))
    p = Pooling.from_sentence_transformers({"word_embedding_dimension": 4, "pooling_mode_mean_tokens": True})
    assert p.strategy == "mean" and p.dimension == 4


def test_embedder_and_cross_encoder():
    m = EncoderModel(_cfg()).init_random(3, std=0.1, num_labels=1)
    emb = Embedder(m).embed([[5, 6, 7], [8, 9, 10, 11]])
    assert emb.shape == (2, 128) and torch.allclose(emb.norm(dim=-1), torch.ones(2), atol=1e-5)
    rr = Reranker(m, cls_id=1, sep_id=2)
    s = rr.score([10, 11, 12], [[20, 21], [30, 31, 32], [10, 11, 12]])
    assert len(s) == 3 and all(0.0 < v < 1.0 for v in s)
    # the score of a document does not depend on its batch-mates
    assert abs(rr.score([10, 11, 12], [[30, 31, 32]])[0] - s[1]) < 1e-5


def test_decoder_embedder_and_reranker():
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(2, std=0.2)
    seqs = [[3, 4, 5, 6], list(range(10, 40))]
    e = Embedder(m).embed(seqs)
    # last-token final-normed hidden of a full forward
    for i, s in enumerate(seqs):
        h = m.forward_dense(torch.tensor(s), m.new_cache(), return_hidden=True)[-1]
        assert torch.allclose(e[i], torch.nn.functional.normalize(h, dim=0), atol=1e-4)
    rr = Reranker(m, yes_no=(7, 9))
    sc = rr.score([1, 2, 3], [[4, 5], [6, 7, 8]])
    lg = m.forward_dense(torch.tensor([1, 2, 3, 6, 7, 8]), m.new_cache())[-1]
    assert abs(sc[1] - torch.softmax(lg[[7, 9]], -1)[1].item()) < 1e-5
    assert RerankScore("binary_margin", positive=1, negative=0, transform="identity")(torch.tensor([[0.5, 2.0]])) \
        == [1.5]
