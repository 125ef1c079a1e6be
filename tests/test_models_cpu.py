"""benchmark config 1 (tiny Qwen3, CPU fp32): paged engine == dense KV path."""
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.engine.types import Request, SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3


def _model(std=0.2, seed=0, **over):
    cfg = tiny_qwen3()
    for k, v in over.items():
        setattr(cfg, k, v)
    return DecoderLM(cfg, "cpu", torch.float32).init_random(seed, std=std)


def _dense_greedy(m, prompt, n):
    c = m.new_cache()
    lg = m.forward_dense(torch.tensor(prompt), c)
    toks, logits = [], [lg[-1]]
    t = int(lg[-1].argmax())
    for _ in range(n):
        toks.append(t)
        lg = m.forward_dense(torch.tensor([t]), c)
        logits.append(lg[-1])
        t = int(lg[-1].argmax())
    return toks, logits


def _engine(m, chunk=16, **kw):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(prefill_chunk_size=chunk, **kw),
                                           max_model_len=512, use_cuda_graphs=False))


def test_paged_equals_dense_tokens_and_logits():
    m = _model()
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, m.cfg.vocab_size, (32,), generator=g).tolist()
    dense_toks, dense_logits = _dense_greedy(m, prompt, 64)
    assert len(set(dense_toks)) > 4, "random model should not be degenerate"
    eng = _engine(m)
    out = eng.generate([prompt], max_tokens=64)[0]
    assert out == dense_toks
    # logits of the paged forward equal the dense ones
    tf = eng.teacher_forced_top1(prompt + dense_toks[:-1])
    assert tf[len(prompt) - 1:] == dense_toks


def test_batch_composition_invariance_cpu():
    m = _model(seed=3)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 17, 33, 40)]
    solo = [_engine(m).generate([p], max_tokens=24)[0] for p in prompts]
    batched = _engine(m, chunk=8).generate(prompts, max_tokens=24)
    assert batched == solo


def test_join_mid_stream_cpu():
    m = _model(seed=4)
    g = torch.Generator().manual_seed(5)
    p1 = torch.randint(0, m.cfg.vocab_size, (20,), generator=g).tolist()
    p2 = torch.randint(0, m.cfg.vocab_size, (11,), generator=g).tolist()
    solo1 = _engine(m).generate([p1], max_tokens=20)[0]
    solo2 = _engine(m).generate([p2], max_tokens=20)[0]
    eng = _engine(m)
    s1 = eng.submit(Request(prompt_tokens=p1, max_tokens=20, sampling=SamplingParams(temperature=0)))
    for _ in range(6):
        eng.step()
    s2 = eng.submit(Request(prompt_tokens=p2, max_tokens=20, sampling=SamplingParams(temperature=0)))
    eng.run_until_idle()
    assert s1.tokens() == solo1
    assert s2.tokens() == solo2


def test_sliding_window_and_sinks_cpu():
    m = _model(seed=6, layer_windows=[8, 0, 8, 0], attention_sinks=True)
    g = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, m.cfg.vocab_size, (30,), generator=g).tolist()
    dense, _ = _dense_greedy(m, prompt, 20)
    assert _engine(m).generate([prompt], max_tokens=20)[0] == dense


def test_seeded_sampling_reproducible_and_batch_invariant():
    m = _model(seed=8)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 12)]
    sp = SamplingParams(temperature=0.8, top_k=50, top_p=0.9, seed=1234)

    def run(ps, ids):
        eng = _engine(m)
        ss = [eng.submit(Request(prompt_tokens=p, max_tokens=16, sampling=sp, id=i)) for p, i in zip(ps, ids)]
        eng.run_until_idle()
        return [s.tokens() for s in ss]

    a = run(prompts, [101, 102])
    b = run(prompts[:1], [101])
    assert a[0] == b[0]
    assert a == run(prompts, [101, 102])
