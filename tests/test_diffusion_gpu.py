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


@pytest.mark.parametrize("R,V,offset", [(64, 151936, 0), (3, 1000, 0), (1, 32, 0), (2, 1001, 0), (3, 151937, 0),
                                        (4, 20000, 1), (300, 16385, 0)])
def test_argmax_confidence_kernel(R, V, offset):
    """V % 4 != 0 runs the scalar tail; an offset view (x[:, 1:]) has an
    unaligned base and row stride, so the scalar path runs for every chunk."""
    torch.manual_seed(V)
    x = (torch.randn(R, V + offset, device=DEV) * 4)[:, offset:]
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


def test_argmax_confidence_independent_of_batch():
    """A row scored alone and inside a batch gets bit-identical results: the
    vocabulary split depends on V only."""
    torch.manual_seed(7)
    V = 151936
    x = torch.randn(300, V, device=DEV) * 3
    tok_b, conf_b, mx_b = ops.argmax_confidence(x)
    for r in (0, 17, 299):
        tok, conf, mx = ops.argmax_confidence(x[r:r + 1].contiguous())
        assert tok.item() == tok_b[r].item()
        assert torch.equal(conf, conf_b[r:r + 1])
        assert torch.equal(mx, mx_b[r:r + 1])
