"""Block mask-diffusion on the GPU: the fused greedy-confidence kernel
against fp32 torch, and batched engine requests against the same requests
run alone (diffusion and linear self-speculation)."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, ops
from mlx_swift_lm_b200.engine.block_diffusion import BlockDiffusionEngine, DiffusionConfig, DiffusionRequest
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("R,V", [(64, 151936), (3, 1000), (1, 32)])
def test_argmax_confidence_kernel(R, V):
    torch.manual_seed(V)
    x = torch.randn(R, V, device=DEV) * 4
    x[0, V // 2] = 40.0
    x[-1, 5] = x[-1, 7] = x[-1].max() + 1.0  # tie -> lower index
    tok, conf, mx = ops.argmax_confidence(x)
    torch.cuda.synchronize()
    assert tok.tolist() == x.argmax(-1).tolist()
    assert tok[-1].item() == 5
    want = torch.softmax(x.double(), -1).max(-1).values.float()
    assert torch.allclose(conf, want, rtol=1e-4, atol=1e-7)
    assert torch.equal(mx, x.max(-1).values)


@pytest.mark.parametrize("mode,thr", [("diffusion", 0.3), ("diffusion", None), ("linear_spec", 0.0)])
def test_engine_batched_equals_single(mode, thr):
    c = tiny_qwen3()
    c.extra["mask_token_id"] = 3
    m = DecoderLM(c, "cuda", torch.bfloat16).init_random(5, std=0.3)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(4, c.vocab_size, (n,), generator=g).tolist() for n in (5, 40, 17, 90)]

    def run(ps):
        eng = BlockDiffusionEngine(m, DiffusionConfig(max_rows=8, prefill_chunk=32, kv_tokens=4096))
        return eng.generate([DiffusionRequest(p, 32, 8, thr, mode) for p in ps])

    both = run(prompts)
    for p, (toks, _) in zip(prompts, both):
        assert run([p])[0][0] == toks
        assert 3 not in toks[len(p):] and len(toks) == len(p) + 32
    assert _lib.read_status().get("sampling", 0) == 0
