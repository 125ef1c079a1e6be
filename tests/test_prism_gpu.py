"""Prism Hadamard path on the GPU: the block Walsh-Hadamard kernel against
the fp32 re-statement, and a packed (2-bit, Hadamard-transformed) hybrid
model through the engine against the same artifact's fp32 CPU forward."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.ops import _lib
from mlx_swift_lm_b200.ops.rotation import HadamardTransform

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("block,K,T", [(512, 1024, 7), (1024, 5120, 3), (4096, 8192, 2), (2, 64, 5)])
def test_block_hadamard_kernel(block, K, T):
    torch.manual_seed(block + T)
    s = (torch.randint(0, 2, (K,)) * 2 - 1).float()
    x = torch.randn(T, K).to(torch.bfloat16)
    tr = HadamardTransform(block, s)
    want = tr.rotate(x.float())
    trd = tr.to(DEV)
    got = trd.rotate(x.to(DEV))
    back = trd.inverse(got)
    torch.cuda.synchronize()
    assert _lib.read_status().get("rotation", 0) == 0
    assert _rel(got.cpu(), want) < 5e-3
    assert _rel(back.cpu(), x.float()) < 1e-2


def test_prism_model_on_gpu(tmp_path):
    from mlx_swift_lm_b200.loader.load import load_model
    from mlx_swift_lm_b200.models.config import tiny_qwen3
    from mlx_swift_lm_b200.testing.prism import write_prism_checkpoint

    c = tiny_qwen3()
    c.model_type = "qwen3_5"
    c.layer_types = ["linear_attention", "linear_attention", "linear_attention", "full_attention"]
    c.attn_output_gate = True
    c.linear_num_key_heads, c.linear_num_value_heads = 2, 4
    c.linear_key_head_dim = c.linear_value_head_dim = 64
    c.tie_word_embeddings = False
    c.hidden_size, c.intermediate_size = 512, 1024
    m = DecoderLM(c, "cpu", torch.float32).init_random(3, std=0.05)
    d = str(tmp_path / "prism")
    write_prism_checkpoint(m, d, block=512)
    cpu, _ = load_model(d, device="cpu", dtype=torch.float32)
    gpu, _ = load_model(d, device="cuda", dtype=torch.bfloat16)
    p = torch.arange(5, 45) % c.vocab_size
    want = cpu.forward_dense(p, cpu.new_cache())
    got = gpu.forward_dense(p.to(DEV), gpu.new_cache()).float().cpu()
    assert _rel(got, want) < 3e-2
    eng = EngineV2(gpu, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                            max_model_len=256, use_cuda_graphs=True))
    out = eng.generate([p.tolist(), p[:11].tolist()], max_tokens=8)
    assert all(len(o) == 8 for o in out)
    assert _lib.read_status().get("rotation", 0) == 0
