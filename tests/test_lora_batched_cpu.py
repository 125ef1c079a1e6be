"""Batched multi-adapter LoRA on CPU: requests naming different adapters (and
none) in one engine batch produce the tokens of the adapter merged into the
weights and served alone; the ops against explicit fp32 math."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.adapters.batched import BatchedLoRA
from mlx_swift_lm_b200.adapters.lora import LoRAConfiguration, LoRAContainer, LoRAParameters
from mlx_swift_lm_b200.engine.types import SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops import lora as lops
from mlx_swift_lm_b200.ops.reference import deinterleave_gate_up

KEYS = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
        "mlp.up_proj", "mlp.down_proj"]


def _adapter(model, seed, rank, keys=KEYS, scale=2.0):
    conf = LoRAConfiguration(num_layers=model.cfg.num_layers,
                             lora_parameters=LoRAParameters(rank=rank, scale=scale, keys=list(keys)))
    ad = LoRAContainer.init_for(model, conf, seed=seed)
    g = torch.Generator().manual_seed(seed + 100)
    for ent in ad.tensors.values():
        ent["b"] = torch.randn(ent["b"].shape, generator=g) * 0.05
    return ad


def _engine(m):
    return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4, prefill_chunk_size=7),
                                           max_model_len=96, use_cuda_graphs=False))


def _run(m, prompt, lora=None, n=10):
    eng = _engine(m)
    s = eng.submit(Request(prompt_tokens=prompt, max_tokens=n, sampling=SamplingParams(temperature=0.0), lora=lora))
    eng.run_until_idle()
    return s.tokens()


def test_batched_adapters_match_merged():
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(5, std=0.1)
    a1, a2 = _adapter(m, 1, 4), _adapter(m, 2, 8, keys=["self_attn.q_proj", "mlp.down_proj"], scale=4.0)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 15, 12)]
    want = []
    for p, ad in zip(prompts, (a1, a2, None)):
        if ad is not None:
            ad.load(m)
        want.append(_run(m, p))
        if ad is not None:
            ad.unload(m)
    assert want[0] != _run(m, prompts[0])  # the adapter changes the output
    m.batched_lora = BatchedLoRA(m, max_adapters=3, max_rank=8)
    m.batched_lora.add("a1", a1)
    m.batched_lora.add("a2", a2)
    eng = _engine(m)
    ss = [eng.submit(Request(prompt_tokens=p, max_tokens=10, sampling=SamplingParams(temperature=0.0), lora=nm))
          for p, nm in zip(prompts, ("a1", "a2", None))]
    eng.run_until_idle()
    assert [s.tokens() for s in ss] == want
    with pytest.raises(ValueError):
        eng.submit(Request(prompt_tokens=[1, 2], max_tokens=2, lora="missing"))
    m.batched_lora.remove("a1")
    assert m.batched_lora.add("a3", a1) == 0  # the freed slot is reused


def test_request_adapter_without_store_is_refused():
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(5)
    with pytest.raises(ValueError):
        _engine(m).submit(Request(prompt_tokens=[1, 2, 3], max_tokens=2, lora="x"))


def test_lora_ops_cpu_math():
    g = torch.Generator().manual_seed(3)
    T, K, R, N, S = 5, 32, 6, 256, 3
    x = torch.randn(T, K, generator=g)
    A = torch.randn(S, R, K, generator=g)
    Bt = torch.randn(S, R, N, generator=g)
    sc = torch.tensor([0.5, 2.0, 1.0])
    slots = torch.tensor([0, -1, 2, 1, 0], dtype=torch.int32)
    t = lops.lora_shrink(x, A, slots)
    y0 = torch.randn(T, N, generator=g)
    y = lops.lora_expand(y0.clone(), Bt, t, slots, sc)
    for i, s in enumerate(slots.tolist()):
        want = y0[i] if s < 0 else y0[i] + sc[s] * (x[i] @ A[s].t()) @ Bt[s]
        assert torch.allclose(y[i], want, atol=1e-4)
    out = lops.lora_expand_glu(y0.clone(), Bt, t, slots, sc, "swiglu")
    pre = y
    gg, uu = deinterleave_gate_up(pre.t())
    assert torch.allclose(out, torch.nn.functional.silu(gg.t()) * uu.t(), atol=1e-4)
