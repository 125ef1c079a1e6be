"""KV compression schemes: codebook quality, rotation inverse, scheme
parsing, attention closeness and memory of compressed legacy caches."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.kv.compress import (CompressedKVCache, _hadamard, lloyd_max_gaussian, parse_scheme,
                                           turbo_dequantize, turbo_quantize, varn_dequantize, varn_quantize)
from mlx_swift_lm_b200.models.config import tiny_qwen3


def test_lloyd_max_levels():
    lv = lloyd_max_gaussian(1)
    assert torch.allclose(lv, torch.tensor([-0.7979, 0.7979]), atol=2e-3)  # +-sqrt(2/pi)
    lv2 = lloyd_max_gaussian(2)
    assert torch.allclose(lv2, torch.tensor([-1.510, -0.4528, 0.4528, 1.510]), atol=3e-3)


def test_rotation_and_turbo_error():
    x = torch.randn(7, 64)
    assert torch.allclose(_hadamard(_hadamard(x)), x, atol=1e-5)
    prev = 1.0
    for b in (2, 3, 4):
        c, n = turbo_quantize(x, b)
        err = ((turbo_dequantize(c, n, b) - x).norm() / x.norm()).item()
        assert err < prev
        prev = err
    assert prev < 0.12


def test_varn_roundtrip():
    x = torch.randn(128, 2, 64) * torch.linspace(0.1, 5, 64) + torch.linspace(-3, 3, 64)
    e = varn_quantize(x, 4)
    err = ((varn_dequantize(*e) - x).norm() / x.norm()).item()
    assert err < 0.1


def test_scheme_parsing():
    assert parse_scheme("turbo8v3") == {"kind": "turbo", "k_bits": 8, "v_bits": 3, "tile": 0}
    assert parse_scheme("turbo4")["v_bits"] == 4
    assert parse_scheme("varn")["k_bits"] == 4 and parse_scheme("varn")["v_bits"] == 2
    assert parse_scheme("varn4v2t32")["tile"] == 32
    with pytest.raises(ValueError):
        parse_scheme("turbo9v9")


def test_compressed_cache_attention():
    """Logit error of the compressed caches (random-init model: no structure
    for the codebooks to exploit, so errors are compared, not absolute):
    TurboQuant's rotated 4-bit values beat plain 4-bit affine, fewer bits
    cost more, 8-bit affine is near lossless, and every scheme is smaller
    than the fp32 cache."""
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(3, std=0.05)
    toks = torch.arange(10, 150)
    ref = m.forward_dense(toks, m.new_cache())
    dense_bytes = 2 * m.cfg.num_layers * len(toks) * m.KVH * m.D * 4
    err = {}
    for scheme in ("affine8", "affine4", "turbo0v4", "turbo0v2", "varn4v4t32", "varn2v2t32"):
        c = CompressedKVCache(m.cfg.num_layers, scheme)
        out = None
        for i in range(0, len(toks), 20):
            out = m.forward_dense(toks[i:i + 20], c)
        err[scheme] = ((out - ref[-20:]).norm() / ref[-20:].norm()).item()
        assert c.nbytes() < dense_bytes, scheme
    assert err["affine8"] < 0.03
    assert err["turbo0v4"] < err["affine4"]
    assert err["turbo0v4"] < err["turbo0v2"] and err["varn4v4t32"] < err["varn2v2t32"]
    assert err["varn4v4t32"] < 1.1 * err["affine4"]
