"""Gated DeltaNet kernels (conv + gates, delta-rule recurrence, gated norm)
against the fp32 oracle, and a hybrid decoder through the engine (graphs vs
eager)."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.ops import _lib
from mlx_swift_lm_b200.ops import reference as ref
from mlx_swift_lm_b200.ops.gdn import GdnRows, gdn_layer, sigmoid_mul

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("Hk,Dk,Hv,Dv", [(2, 128, 4, 128), (4, 64, 4, 64), (1, 256, 2, 128)])
def test_gdn_layer_matches_oracle(Hk, Dk, Hv, Dv):
    torch.manual_seed(Dk + Hv)
    C = 2 * Hk * Dk + Hv * Dv
    lens = [1, 1, 1, 37, 2, 300]  # three decode rows, then prefill chunks
    fresh = [0, 0, 0, 1, 0, 0]
    slots = [5, 0, 3, 1, 2, 4]
    T = sum(lens)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    P = (torch.randn(T, C + Hv * Dv + 2 * Hv) * 0.5).to(torch.bfloat16)
    conv_w = torch.randn(C, 4) * 0.5
    A_log, dt_bias = torch.rand(Hv) * 2, torch.randn(Hv)
    norm_w = (torch.rand(Dv) + 0.5).to(torch.bfloat16)
    S = 6
    cs0 = (torch.randn(S, 3, C) * 0.5).to(torch.bfloat16)
    ss0 = torch.randn(S, Hv, Dv, Dk) * 0.1
    cs_r, ss_r = cs0.clone(), ss0.clone()
    want = ref.gdn_layer_ref(P.float(), cu, fresh, slots, cs_r, ss_r, conv_w, A_log, dt_bias, norm_w.float(),
                             Hk, Dk, Hv, Dv, 1e-6)
    i32 = dict(dtype=torch.int32, device=DEV)
    rows = GdnRows(torch.tensor(cu, **i32), torch.tensor(fresh, **i32), torch.tensor(slots, **i32), cu)
    cs, ss = cs0.to(DEV), ss0.to(DEV)
    got = gdn_layer(P.to(DEV), rows, cs, ss, conv_w.to(DEV), A_log.to(DEV), dt_bias.to(DEV), norm_w.to(DEV),
                    Hk, Dk, Hv, Dv, 1e-6)
    torch.cuda.synchronize()
    assert _lib.read_status().get("gdn", 0) == 0
    assert _rel(got.cpu(), want) < 1e-2
    assert _rel(ss.cpu(), ss_r) < 1e-4
    assert torch.equal(cs.cpu(), cs_r.to(torch.bfloat16))


def test_sigmoid_mul():
    x = torch.randn(33, 96, device=DEV, dtype=torch.bfloat16)
    g = torch.randn(33, 200, device=DEV, dtype=torch.bfloat16)[:, 50:146]
    y = sigmoid_mul(x, g)
    r = (x.float() * torch.sigmoid(g.float())).to(torch.bfloat16)
    assert _rel(y, r) < 1e-2


def _hybrid(seed=0):
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    c = tiny_qwen3()
    c.model_type = "qwen3_next"
    c.layer_types = ["linear_attention", "full_attention", "linear_attention", "full_attention"]
    c.attn_output_gate = True
    c.linear_num_key_heads, c.linear_num_value_heads = 2, 4
    c.linear_key_head_dim = c.linear_value_head_dim = 128
    return DecoderLM(c, DEV, torch.bfloat16).init_random(seed, std=0.2)


def test_hybrid_model_graph_matches_eager_and_oracle():
    m = _hybrid()
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=16) == eng(False).generate(ps, max_tokens=16)
    p = torch.tensor(ps[1])
    lg = m.forward_dense(p.to(DEV), m.new_cache()).float().cpu()
    mc = m.clone_to("cpu", torch.float32)
    r = mc.forward_dense(p, mc.new_cache())
    assert _rel(lg, r) < 0.05


@pytest.mark.parametrize("Dk", [64, 128])
def test_gdn_decode_rows_four_per_warp(Dk):
    """A decode batch large enough for the several-rows-per-warp kernel."""
    torch.manual_seed(Dk)
    Hk, Hv, Dv, B = 2, 8, 128, 48
    C = 2 * Hk * Dk + Hv * Dv
    P = (torch.randn(B, C + Hv * Dv + 2 * Hv) * 0.5).to(torch.bfloat16)
    conv_w = torch.randn(C, 4) * 0.5
    A_log, dt_bias = torch.rand(Hv) * 2, torch.randn(Hv)
    norm_w = (torch.rand(Dv) + 0.5).to(torch.bfloat16)
    cs0 = (torch.randn(B + 1, 3, C) * 0.5).to(torch.bfloat16)
    ss0 = torch.randn(B + 1, Hv, Dv, Dk) * 0.1
    cu, fresh, slots = list(range(B + 1)), [0] * B, list(range(B))
    cs_r, ss_r = cs0.clone(), ss0.clone()
    want = ref.gdn_layer_ref(P.float(), cu, fresh, slots, cs_r, ss_r, conv_w, A_log, dt_bias, norm_w.float(),
                             Hk, Dk, Hv, Dv, 1e-6)
    i32 = dict(dtype=torch.int32, device=DEV)
    rows = GdnRows(torch.tensor(cu, **i32), torch.tensor(fresh, **i32), torch.tensor(slots, **i32))
    cs, ss = cs0.to(DEV), ss0.to(DEV)
    got = gdn_layer(P.to(DEV), rows, cs, ss, conv_w.to(DEV), A_log.to(DEV), dt_bias.to(DEV), norm_w.to(DEV),
                    Hk, Dk, Hv, Dv, 1e-6)
    torch.cuda.synchronize()
    assert _rel(got.cpu(), want) < 1e-2
    assert _rel(ss.cpu(), ss_r) < 1e-4
