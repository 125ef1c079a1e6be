"""Encoder path on the GPU: GELU epilogues, fused residual + LayerNorm,
bidirectional tensor-core attention, and a BERT-style encoder against its
fp32 CPU oracle."""
import pytest
import torch

from mlx_swift_lm_b200 import ops
from mlx_swift_lm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("epi", ["gelu", "gelu_tanh"])
def test_gemm_gelu_epilogue(epi):
    torch.manual_seed(1)
    x = torch.randn(40, 384, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(1536, 384, device=DEV, dtype=torch.bfloat16) * 0.05
    b = torch.randn(1536, device=DEV, dtype=torch.bfloat16) * 0.1
    y = ops.gemm(x, w, epi=epi, bias=b)
    assert _rel(y.cpu(), ref.gemm_ref(x.cpu(), w.cpu(), epi, bias=b.cpu())) < 1e-2


def test_add_layernorm():
    torch.manual_seed(2)
    x = torch.randn(17, 768, device=DEV, dtype=torch.bfloat16)
    d = torch.randn(17, 768, device=DEV, dtype=torch.bfloat16)
    w = torch.rand(768, device=DEV, dtype=torch.bfloat16) + 0.5
    b = torch.randn(768, device=DEV, dtype=torch.bfloat16) * 0.1
    xc, dc = x.cpu().float(), d.cpu().float()
    s = (xc + dc).to(torch.bfloat16).float()
    want = torch.nn.functional.layer_norm(s, (768,), w.cpu().float(), b.cpu().float(), 1e-12)
    y = ops.add_layernorm(x, d, w, b, 1e-12, out=x)  # in place, as the encoder uses it
    assert _rel(y.cpu(), want) < 1e-2


def test_bidirectional_paged_prefill():
    torch.manual_seed(3)
    H, D, P = 4, 64, 16
    lens = [5, 70, 33]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T = cu[-1]
    npg = [(n + P - 1) // P for n in lens]
    kc = torch.randn(sum(npg) + 1, H, P, D, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    pt = torch.zeros(len(lens), max(npg), dtype=torch.int32)
    p = 1
    for r, k in enumerate(npg):
        pt[r, :k] = torch.arange(p, p + k)
        p += k
    q = torch.randn(T, H, D, dtype=torch.bfloat16)
    cu_t, p0 = torch.tensor(cu, dtype=torch.int32), torch.zeros(len(lens), dtype=torch.int32)
    want = ref.paged_prefill_ref(q, kc, vc, pt, cu_t, p0, D ** -0.5, -1)
    got = ops.paged_prefill(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), cu_t.to(DEV), p0.to(DEV), D ** -0.5, -1,
                            cu_q_host=cu)
    assert _rel(got.cpu(), want) < 1e-2


def test_encoder_matches_cpu_oracle():
    from mlx_swift_lm_b200.api.embed import Embedder
    from mlx_swift_lm_b200.models.encoder import EncoderConfig, EncoderModel

    for kw in ({}, {"rotary": True, "hidden_act": "swiglu", "bias": False}):
        cfg = EncoderConfig(vocab_size=1000, hidden_size=256, num_layers=2, num_heads=4, intermediate_size=1024,
                            max_position_embeddings=256)
        for k, v in kw.items():
            setattr(cfg, k, v)
        m = EncoderModel(cfg).init_random(4, std=0.05)
        seqs = [list(range(5, 40)), list(range(100, 300)), [7, 8, 9]]
        e_cpu = Embedder(m).embed(seqs)
        mg = m.to(DEV, torch.bfloat16)
        e_gpu = Embedder(mg).embed(seqs)
        cos = torch.nn.functional.cosine_similarity(e_gpu.cpu(), e_cpu, dim=-1)
        assert (cos > 0.999).all(), (kw, cos)
