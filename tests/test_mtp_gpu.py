"""MTP rounds on the GPU: the captured fixed-geometry round (draft window,
draft steps, verify as decode rows, device accept walk in one CUDA graph)
emits exactly the tokens of plain greedy graph decoding, and under the
Bernoulli schedule matches the same round run without graphs."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.mtp import MTPConfig
from mlx_swift_lm_b200.engine.types import Request, SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.models.mtp import MTPModule
from mlx_swift_lm_b200.ops import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _eng(m, graphs=True):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=64),
                                           max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))


def _run(eng, ps, n=30):
    ss = [eng.submit(Request(prompt_tokens=p, max_tokens=n, sampling=SamplingParams(temperature=0.0),
                             ignore_eos=True)) for p in ps]
    eng.run_until_idle()
    return [s.tokens() for s in ss]


def _setup():
    m = DecoderLM(tiny_qwen3(), DEV, torch.bfloat16).init_random(0, std=0.05)
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 77)]
    return m, ps


def test_graph_round_equals_plain_greedy():
    m, ps = _setup()
    ref = _run(_eng(m), ps)
    eng = _eng(m)
    drv = eng.enable_mtp(MTPModule(m).init_random(3, std=0.05), MTPConfig(k=3))
    assert drv.runner is not None and drv.runner.use_graphs
    assert _run(eng, ps) == ref
    assert drv.stats.rounds > 0 and any(R.graph is not None for R in drv.runner.rounds.values())
    assert _lib.read_status().get("mtp", 0) == 0


def test_graph_round_bernoulli_equals_ungraphed():
    m, ps = _setup()
    out = []
    for graphs in (False, True):
        eng = _eng(m, graphs)
        drv = eng.enable_mtp(MTPModule(m).init_random(3, std=0.05),
                             MTPConfig(k=3, acceptance="bernoulli", p=0.7, seed=2))
        out.append((_run(eng, ps), drv.stats.accepted, drv.stats.rounds))
    assert out[0] == out[1] and out[1][1] > 0
