"""Prefix-cache tiers: a block evicted from the device goes to the pinned
host tier and a later match restores it into fresh pages (same tokens as
recomputing); save / load of the cache carries warm prefixes into a new
engine; a checkpoint of another geometry is refused."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _model():
    return DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(0, std=0.2)


def _engine(m, **kw):
    cfg = dict(scheduler=SchedulerConfig(max_concurrent_requests=2, prefill_chunk_size=64), max_model_len=256,
               use_cuda_graphs=False, enable_prefix_cache=True, prefix_block_size=32)
    cfg.update(kw)
    return EngineV2(m, config=EngineConfig(**cfg))


def test_host_tier_restores_evicted_blocks():
    m = _model()
    g = torch.Generator().manual_seed(1)
    shared = torch.randint(0, 300, (100,), generator=g).tolist()
    a = shared + [7, 8, 9]
    b = shared + [11, 12]
    want = _engine(m, enable_prefix_cache=False).generate([b], max_tokens=6)
    e = _engine(m, kv_tokens=256, prefix_host_blocks=64)
    e.generate([a], max_tokens=6)
    assert e.prefix_cache.num_blocks == 3
    # unrelated long requests push the shared blocks out of the small device pool
    for s in range(3):
        e.generate([torch.randint(0, 300, (200,), generator=g).tolist()], max_tokens=4)
    assert e.prefix_cache.host.stores > 0
    got = e.generate([b], max_tokens=6)
    assert got == want
    assert e.prefix_cache.host_hits > 0


def test_save_load_warm_start(tmp_path):
    m = _model()
    g = torch.Generator().manual_seed(2)
    shared = torch.randint(0, 300, (70,), generator=g).tolist()
    e = _engine(m)
    e.generate([shared + [1, 2, 3]], max_tokens=5)
    assert e.prefix_cache.save(str(tmp_path / "pc")) == 2
    e2 = _engine(m)
    assert e2.prefix_cache.load(str(tmp_path / "pc")) == 2
    want = _engine(m, enable_prefix_cache=False).generate([shared + [4, 5]], max_tokens=6)
    got = e2.generate([shared + [4, 5]], max_tokens=6)
    assert got == want and e2.prefix_cache.hits == 1 and e2.prefix_cache.hit_tokens == 64
    e3 = _engine(m, prefix_block_size=64)
    with pytest.raises(ValueError):
        e3.prefix_cache.load(str(tmp_path / "pc"))
