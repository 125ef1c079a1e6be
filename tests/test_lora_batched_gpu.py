"""Batched multi-adapter LoRA kernels on the GPU against the fp32 CPU
statements, and a mixed adapter / no-adapter batch through the engine with
CUDA graphs equal to the eager engine."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.adapters.batched import BatchedLoRA
from mlx_swift_lm_b200.adapters.lora import LoRAConfiguration, LoRAContainer, LoRAParameters
from mlx_swift_lm_b200.engine.types import SamplingParams
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops import _lib
from mlx_swift_lm_b200.ops import lora as lops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("T,K,R,N,act", [(1, 4096, 16, 6144, "swiglu"), (37, 2048, 48, 1024, "geglu"),
                                         (64, 4096, 8, 24576, "swiglu_oai")])
def test_lora_kernels_match_cpu(T, K, R, N, act):
    g = torch.Generator().manual_seed(T)
    S = 3
    x = (torch.randn(T, K, generator=g) * 0.5).bfloat16()
    A = (torch.randn(S, R, K, generator=g) * 0.05).bfloat16()
    Bt = (torch.randn(S, R, N, generator=g) * 0.05).bfloat16()
    sc = torch.tensor([0.5, 2.0, 1.0])
    slots = torch.randint(-1, S, (T,), generator=g, dtype=torch.int32)
    y0 = (torch.randn(T, N, generator=g)).bfloat16()
    t_ref = lops.lora_shrink(x.float(), A.float(), slots)
    t = lops.lora_shrink(x.to(DEV), A.to(DEV), slots.to(DEV))
    torch.testing.assert_close(t.cpu(), t_ref, atol=2e-3, rtol=2e-3)
    y_ref = lops.lora_expand(y0.float().clone(), Bt.float(), t_ref, slots, sc)
    y = lops.lora_expand(y0.to(DEV).clone(), Bt.to(DEV), t, slots.to(DEV), sc.to(DEV))
    torch.testing.assert_close(y.float().cpu(), y_ref, atol=3e-2, rtol=2e-2)
    o_ref = lops.lora_expand_glu(y0.clone(), Bt, t_ref, slots, sc, act).float()
    o = lops.lora_expand_glu(y0.to(DEV), Bt.to(DEV), t, slots.to(DEV), sc.to(DEV), act)
    torch.testing.assert_close(o.float().cpu(), o_ref, atol=3e-2, rtol=3e-2)
    assert _lib.read_status().get("lora", 0) == 0


def _adapter(model, seed, rank, scale=2.0):
    keys = ["self_attn.q_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj",
            "mlp.down_proj"]
    conf = LoRAConfiguration(num_layers=model.cfg.num_layers,
                             lora_parameters=LoRAParameters(rank=rank, scale=scale, keys=keys))
    ad = LoRAContainer.init_for(model, conf, seed=seed)
    g = torch.Generator().manual_seed(seed + 100)
    for ent in ad.tensors.values():
        ent["b"] = torch.randn(ent["b"].shape, generator=g) * 0.05
    return ad


def test_engine_graphs_with_adapters_equal_eager():
    m = DecoderLM(tiny_qwen3(), DEV, torch.bfloat16).init_random(5, std=0.05)
    m.batched_lora = BatchedLoRA(m, max_adapters=2, max_rank=8)
    m.batched_lora.add("a", _adapter(m, 1, 8))
    m.batched_lora.add("b", _adapter(m, 2, 4, scale=4.0))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 30, 17, 5)]
    names = ["a", None, "b", "a"]

    def run(graphs):
        eng = EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                              max_model_len=128, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))
        ss = [eng.submit(Request(prompt_tokens=p, max_tokens=12, sampling=SamplingParams(temperature=0.0), lora=n))
              for p, n in zip(prompts, names)]
        eng.run_until_idle()
        return [s.tokens() for s in ss], eng

    eager, _ = run(False)
    graphed, eng = run(True)
    assert graphed == eager
    assert eng.graphs is not None and eng.graphs.lgraphs  # the LoRA variant ran
    base = DecoderLM(tiny_qwen3(), DEV, torch.bfloat16).init_random(5, std=0.05)
    e2 = EngineV2(base, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4), max_model_len=128,
                                            use_cuda_graphs=False))
    s = e2.submit(Request(prompt_tokens=prompts[1], max_tokens=12, sampling=SamplingParams(temperature=0.0)))
    e2.run_until_idle()
    assert s.tokens() == eager[1]  # the row without an adapter is the base model
