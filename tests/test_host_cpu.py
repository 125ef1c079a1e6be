"""Host-side runtime: page pool, block hashing, prefix cache, scheduler,
detokenizer / stop holdback, quant codecs, safetensors round trip."""
import hashlib
import struct

import numpy as np
import pytest
import torch

from mlx_swift_lm_b200.engine.detok import IncrementalDetokenizer, StopHoldback
from mlx_swift_lm_b200.engine.scheduler import Scheduler, SchedulerConfig, Status
from mlx_swift_lm_b200.engine.types import Request
from mlx_swift_lm_b200.kv.paged import PagedKVCache, _b200host
from mlx_swift_lm_b200.ops import quant
from mlx_swift_lm_b200.ops import reference as ref


def test_page_pool_refcounts_generations_poison():
    p = _b200host.PagePool(8)
    a = p.alloc(3)
    assert p.num_free == 5
    g0 = p.generation(a[0])
    p.incref([a[0]])
    assert p.decref(a) == 2 and p.refcount(a[0]) == 1
    assert p.valid(a[0], g0)
    p.decref([a[0]])
    assert not p.valid(a[0], g0)
    with pytest.raises(RuntimeError):
        p.decref([a[0]])
    b = p.alloc(2)
    p.poison(b[0])
    p.decref(b)
    assert p.num_poisoned == 1 and p.num_free == 7
    with pytest.raises(RuntimeError):
        p.alloc(8)


def test_block_hash_chain_matches_hashlib():
    toks = list(range(100, 164))
    hs = _b200host.block_hashes(toks, 16, "salt")
    prev = b"salt"
    for i in range(4):
        d = hashlib.sha256(prev + struct.pack("<16i", *toks[i * 16:(i + 1) * 16])).digest()
        assert d == hs[i]
        prev = d
    assert _b200host.block_hashes(toks, 16, "other")[0] != hs[0]
    assert len(_b200host.block_hashes(toks[:40], 16, "")) == 2


def _sched(pages=64, **kw):
    cache = PagedKVCache(1, pages, 1, 8, torch.float32, "cpu")
    return Scheduler(SchedulerConfig(**kw), cache), cache


def test_scheduler_chunked_prefill_and_budget():
    s, _ = _sched(max_batched_tokens_per_step=40, prefill_chunk_size=16)
    a = s.add(Request(prompt_tokens=list(range(50)), max_tokens=4))
    b = s.add(Request(prompt_tokens=list(range(10)), max_tokens=4))
    plan = s.plan()
    assert [(r.state is a, r.num_tokens) for r in plan.rows] == [(True, 16), (False, 10)]
    for r in plan.rows:
        s.commit(r)
    plan = s.plan()
    assert plan.rows[0].state is a and plan.rows[0].num_tokens == 16
    assert sum(r.num_tokens for r in plan.rows) <= 40


def test_scheduler_priority_and_preemption():
    s, cache = _sched(pages=6, max_batched_tokens_per_step=256, prefill_chunk_size=256)
    lo = s.add(Request(prompt_tokens=list(range(40)), max_tokens=40, priority=0))
    plan = s.plan()
    for r in plan.rows:
        s.commit(r)
    lo.all_tokens.append(1)
    hi = s.add(Request(prompt_tokens=list(range(40)), max_tokens=4, priority=5))
    plan = s.plan()  # hi cannot fit alongside lo: waits (FCFS head of line)
    assert lo in [r.state for r in plan.rows]
    for r in plan.rows:
        s.commit(r)
    # grow lo until the pool is exhausted: lo is preempted when it cannot grow
    while lo.status == Status.RUNNING:
        lo.all_tokens.append(2)
        plan = s.plan()
        for r in plan.rows:
            s.commit(r)
        if plan.preempted:
            break
    assert lo.status == Status.WAITING and lo.timing.preemptions == 1
    assert lo.seq.num_tokens == 0


def test_prefix_cache_reuse_and_eviction():
    from mlx_swift_lm_b200.kv.prefix_cache import PrefixCache

    cache = PagedKVCache(1, 32, 1, 8, torch.float32, "cpu")
    pc = PrefixCache(cache, block_size=32)
    s = Scheduler(SchedulerConfig(prefill_chunk_size=512), cache, pc)
    a = s.add(Request(prompt_tokens=list(range(70)), max_tokens=1))
    for r in s.plan().rows:
        s.commit(r)
    pc.donate(a)
    s.finish(a)
    a.seq.release()
    assert pc.num_blocks == 2
    b = s.add(Request(prompt_tokens=list(range(70)) + [5, 6], max_tokens=1))
    plan = s.plan()
    assert b.usage.cached_prompt_tokens == 64 and plan.rows[0].start == 64
    c = s.add(Request(prompt_tokens=list(range(70)), max_tokens=1, cache_salt="tenant-b"))
    s.plan()
    assert c.usage.cached_prompt_tokens == 0
    freed = pc.evict(100)
    assert freed == 0  # pages still held by b
    b.seq.release()
    assert pc.evict(100) == 4


def test_detokenizer_utf8_and_stop_holdback():
    from mlx_swift_lm_b200.api.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    d = IncrementalDetokenizer(tok)
    ids = tok.encode("héllo wörld")
    out = "".join(d.push([t]) for t in ids) + d.flush()
    assert out == "héllo wörld"
    h = StopHoldback(["STOP", "</end>"])
    emitted = []
    stopped = False
    for piece in ["hello S", "TO", "P tail"]:
        t, stopped = h.push(piece)
        emitted.append(t)
        if stopped:
            break
    assert "".join(emitted) == "hello " and stopped


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_affine_quant_roundtrip(bits):
    torch.manual_seed(bits)
    w = torch.randn(16, 128)
    q, s, b = quant.affine_quantize(w, 64, bits)
    assert q.shape == (16, 128 * bits // 32)
    wd = quant.affine_dequantize(q, s, b, 64, bits)
    err = (wd - w).abs().max() / w.abs().max()
    assert err < 2.0 / (2 ** bits - 1) + 1e-3
    codes = quant.unpack_codes(quant.pack_codes(torch.randint(0, 2 ** bits, (4, 64)), bits), bits, 64)
    assert codes.shape == (4, 64)


def test_mxfp4_roundtrip():
    torch.manual_seed(0)
    w = torch.randn(8, 64)
    q, s = quant.mxfp4_quantize(w)
    wd = quant.mxfp4_dequantize(q, s)
    assert ((wd - w).abs() / (w.abs().max())).max() < 0.25


def test_safetensors_roundtrip(tmp_path):
    from mlx_swift_lm_b200.loader.safetensors import load_safetensors, save_safetensors

    t = {"a": torch.randn(3, 5), "b": torch.arange(10, dtype=torch.int32), "c": torch.randn(4).to(torch.bfloat16)}
    p = str(tmp_path / "x.safetensors")
    save_safetensors(p, t, {"format": "pt"})
    back, meta = load_safetensors(p)
    assert meta["format"] == "pt"
    for k in t:
        assert torch.equal(back[k], t[k])


def test_philox_reference_is_deterministic():
    a = ref.philox_u32(1, 2, np.arange(8))
    b = ref.philox_u32(1, 2, np.arange(8))
    assert (a == b).all() and len(set(a.tolist())) == 8
    u = ref.philox_uniform(5, 0, np.arange(10000))
    assert 0 < u.min() and u.max() < 1 and abs(u.mean() - 0.5) < 0.02


def test_sampling_oracle_semantics():
    lg = torch.tensor([5.0, 4.0, 3.0, 2.0, 1.0, 0.0])
    assert ref.sample_ref(lg, 0.0) == 0
    toks = {ref.sample_ref(lg, 1.0, top_k=2, key=k) for k in range(200)}
    assert toks <= {0, 1} and len(toks) == 2
    toks = {ref.sample_ref(lg, 1.0, top_p=0.5, key=k) for k in range(200)}
    assert toks == {0}
    toks = {ref.sample_ref(lg, 1.0, min_p=0.3, key=k) for k in range(300)}
    assert toks <= {0, 1}
    p = ref.process_logits_ref(torch.tensor([1.0, -1.0, 2.0]), {0: 1.0}, [1, 1, 2], 2.0, [2, 2], 0.5, 0.25)
    assert torch.allclose(p, torch.tensor([2.0, -2.0, 1.0 - 1.25]))
