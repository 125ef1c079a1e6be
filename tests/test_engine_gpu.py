"""Engine on the GPU: graph decode == eager decode, batch invariance, and
agreement of the bf16 CUDA forward with the fp32 CPU oracle forward."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.types import Request, SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _model(seed=0, std=0.2, **over):
    cfg = tiny_qwen3()
    for k, v in over.items():
        setattr(cfg, k, v)
    return DecoderLM(cfg, DEV, torch.bfloat16).init_random(seed, std=std)


def _eng(m, graphs=True, chained=True, chunk=64, buckets=(1, 2, 4, 8)):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=8,
                                                                     prefill_chunk_size=chunk),
                                           max_model_len=512, use_cuda_graphs=graphs, chained_decode=chained,
                                           graph_buckets=buckets))


def _prompts(vocab, lens, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


def test_graph_decode_matches_eager():
    m = _model()
    ps = _prompts(m.cfg.vocab_size, (31, 7, 64, 100))
    eager = _eng(m, graphs=False).generate(ps, max_tokens=40)
    graph = _eng(m, graphs=True, chained=False).generate(ps, max_tokens=40)
    chained = _eng(m, graphs=True, chained=True).generate(ps, max_tokens=40)
    assert graph == eager
    assert chained == eager


def test_batch_invariance_gpu():
    m = _model(seed=2)
    ps = _prompts(m.cfg.vocab_size, (5, 17, 33, 140, 260), seed=3)
    solo = [_eng(m).generate([p], max_tokens=32)[0] for p in ps]
    batched = _eng(m, chunk=48).generate(ps, max_tokens=32)
    assert batched == solo


def test_windows_and_sinks_gpu_vs_cpu():
    m = _model(seed=4, layer_windows=[8, 0, 8, 0], attention_sinks=True)
    ps = _prompts(m.cfg.vocab_size, (40, 12), seed=5)
    eng = _eng(m)
    out = eng.generate(ps, max_tokens=8)
    mc = m.clone_to("cpu", torch.float32)
    cpu = EngineV2(mc, config=EngineConfig(max_model_len=512, use_cuda_graphs=False)).generate(ps, max_tokens=8)
    agree = sum(a == b for x, y in zip(out, cpu) for a, b in zip(x, y)) / 16
    assert agree >= 0.75, (out, cpu)


def test_gpu_logits_close_to_cpu_oracle():
    m = _model(seed=6)
    p = _prompts(m.cfg.vocab_size, (48,), seed=7)[0]
    eng = _eng(m)
    from mlx_swift_lm_b200.models.batch import ForwardBatch

    st = eng.sched.add(Request(prompt_tokens=p, max_tokens=1))
    eng.sched.waiting.remove(st)
    st.seq.ensure(len(p))
    fb = ForwardBatch(input_ids=torch.tensor(p, dtype=torch.int32, device=DEV),
                      positions=torch.arange(len(p), dtype=torch.int32, device=DEV),
                      slots=torch.tensor(st.seq.slots(0, len(p)), dtype=torch.int64, device=DEV),
                      pf_cu_q=torch.tensor([0, len(p)], dtype=torch.int32, device=DEV), pf_cu_q_host=[0, len(p)],
                      pf_pos0=torch.tensor([0], dtype=torch.int32, device=DEV),
                      pf_page_table=torch.tensor([st.seq.pages], dtype=torch.int32, device=DEV))
    lg = m.forward(fb, eng.kv).cpu()
    mc = m.clone_to("cpu", torch.float32)
    ref = mc.forward_dense(torch.tensor(p), mc.new_cache())
    rel = ((lg - ref).norm() / ref.norm()).item()
    assert rel < 0.05, rel


def test_seeded_sampling_gpu_matches_cpu_rule():
    m = _model(seed=8)
    ps = _prompts(m.cfg.vocab_size, (20, 33), seed=9)
    sp = SamplingParams(temperature=0.9, top_k=64, top_p=0.95, seed=77)
    e1, e2 = _eng(m), _eng(m)
    s1 = [e1.submit(Request(prompt_tokens=p, max_tokens=12, sampling=sp, id=900 + i)) for i, p in enumerate(ps)]
    e1.run_until_idle()
    s2 = [e2.submit(Request(prompt_tokens=ps[0], max_tokens=12, sampling=sp, id=900))]
    e2.run_until_idle()
    assert s1[0].tokens() == s2[0].tokens()


def test_graph_sampled_decode_matches_eager():
    """Temperature / top-k / top-p / min-p rows run the sampled decode graph
    (chained); under the same seeds they draw exactly the tokens the eager
    sampler draws, mixed with greedy rows in the same batch."""
    m = _model(seed=4, std=0.3)
    ps = _prompts(m.cfg.vocab_size, (12, 40, 7, 90), seed=5)
    sps = [SamplingParams(temperature=0.8, top_p=0.9, seed=11), SamplingParams(temperature=0.0),
           SamplingParams(temperature=1.2, top_k=50, seed=12), SamplingParams(temperature=0.7, min_p=0.05, seed=13)]

    def run(graphs, chained=True):
        eng = _eng(m, graphs=graphs, chained=chained)
        # the RNG key mixes the seed with the request id: pin the ids
        ss = [eng.submit(Request(prompt_tokens=p, max_tokens=30, sampling=sp, id=9000 + i))
              for i, (p, sp) in enumerate(zip(ps, sps))]
        eng.run_until_idle()
        return [s.tokens() for s in ss], eng

    eager, _ = run(False)
    graph, eng = run(True)
    assert eng.graphs.sgraphs, "sampled rows did not use a sampled graph"
    assert graph == eager
    assert run(True, chained=False)[0] == eager
