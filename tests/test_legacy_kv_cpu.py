"""Legacy single-sequence caches: rotating window, quantised, chunked,
prompt-cache files (CPU, fp32)."""
import torch

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.kv.legacy import (ChunkedKVCache, QuantizedKVCache, RotatingKVCache, load_prompt_cache,
                                         save_prompt_cache)
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _m():
    return DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(3, std=0.2)


def _run(m, cache, toks, chunk=5):
    out = None
    for i in range(0, len(toks), chunk):
        out = m.forward_dense(torch.tensor(toks[i:i + chunk]), cache)
    return out


def test_rotating_matches_dense_inside_window_and_keeps_sinks():
    m = _m()
    L = m.cfg.num_layers
    toks = list(range(10, 40))
    a = _run(m, RotatingKVCache(L, max_size=64), toks)
    b = _run(m, m.new_cache(), toks)
    assert torch.allclose(a, b, atol=1e-5)
    c = RotatingKVCache(L, max_size=16, keep=4)
    _run(m, c, toks)
    assert c.k[0].shape[0] == 16
    assert c.pos[0].tolist() == [0, 1, 2, 3] + list(range(18, 30))


def test_quantized_cache_close_to_dense_and_smaller():
    m = _m()
    toks = list(range(10, 50))
    q = QuantizedKVCache(m.cfg.num_layers, bits=8, group_size=32)
    a = _run(m, q, toks)
    b = _run(m, m.new_cache(), toks)
    assert ((a - b).norm() / b.norm()).item() < 2e-2
    dense_bytes = 2 * m.cfg.num_layers * len(toks) * m.KVH * m.D * 4
    assert q.nbytes() < dense_bytes / 2
    q.trim(5)
    assert q.offset == len(toks) - 5 and q.pos[0].shape[0] == len(toks) - 5


def test_chunked_cache_keeps_current_chunk():
    m = _m()
    c = ChunkedKVCache(m.cfg.num_layers, chunk_size=8)
    _run(m, c, list(range(10, 30)), chunk=4)
    assert c.pos[0].tolist() == list(range(16, 20))
    qp, kp = torch.tensor([17]), torch.arange(20)
    assert c.chunk_mask(qp, kp)[0].tolist() == [False] * 16 + [True] * 4


def test_prompt_cache_roundtrip(tmp_path):
    m = _m()
    toks = list(range(10, 40))
    for make in (lambda: m.new_cache(), lambda: RotatingKVCache(m.cfg.num_layers, 16),
                 lambda: QuantizedKVCache(m.cfg.num_layers, 8, 32)):
        c = make()
        _run(m, c, toks)
        p = str(tmp_path / "pc.safetensors")
        save_prompt_cache(p, c, {"model": "tiny"})
        c2, md = load_prompt_cache(p)
        assert md["model"] == "tiny" and c2.offset == c.offset and type(c2) is type(c)
        nxt = torch.tensor([7])
        assert torch.allclose(m.forward_dense(nxt, c), m.forward_dense(nxt, c2), atol=1e-6)
