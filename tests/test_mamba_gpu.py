"""Mamba-2 mixers on the GPU: the conv / SSM / gated-group-norm kernels
(mode 1 of the recurrent kernels) against the fp32 oracle for prefill
chunks and decode rows (including the several-rows-per-warp decode path),
the relu^2 GEMM epilogue, and a NemotronH-style hybrid through the engine
(graphs vs eager, and against the fp32 CPU forward)."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig, ops
from mlx_swift_lm_b200.models.families import build_config
from mlx_swift_lm_b200.ops import _lib
from mlx_swift_lm_b200.ops import reference as ref
from mlx_swift_lm_b200.ops.gdn import GdnRows, mamba_layer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("G,N,H,Pd,lens", [(2, 128, 8, 64, [1, 1, 1, 37, 2, 300]), (1, 64, 4, 32, [5, 1, 90]),
                                           (8, 128, 64, 64, [1] * 48), (1, 256, 4, 64, [1, 17])])
def test_mamba_layer_matches_oracle(G, N, H, Pd, lens):
    torch.manual_seed(N + H)
    C = 2 * G * N + H * Pd
    R = len(lens)
    fresh = [i % 3 == 1 for i in range(R)]
    slots = list(range(R))[::-1]
    T = sum(lens)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    P = (torch.randn(T, C + H * Pd + H) * 0.5).to(torch.bfloat16)
    conv_w, conv_b = torch.randn(C, 4) * 0.5, torch.randn(C) * 0.1
    A_log, dt_bias, D = torch.rand(H) * 2, torch.randn(H), torch.randn(H)
    norm_w = (torch.rand(H * Pd) + 0.5).to(torch.bfloat16)
    cs0 = (torch.randn(R, 3, C) * 0.5).to(torch.bfloat16)
    ss0 = torch.randn(R, H, Pd, N) * 0.1
    cs_r, ss_r = cs0.clone(), ss0.clone()
    lim = (0.0, 4.0)
    want = ref.mamba_layer_ref(P.float(), cu, [int(f) for f in fresh], slots, cs_r, ss_r, conv_w, conv_b, A_log,
                               dt_bias, D, norm_w.float(), G, N, H, Pd, 1e-5, H * Pd // G, lim)
    i32 = dict(dtype=torch.int32, device=DEV)
    rows = GdnRows(torch.tensor(cu, **i32), torch.tensor([int(f) for f in fresh], **i32), torch.tensor(slots, **i32),
                   cu)
    cs, ss = cs0.to(DEV), ss0.to(DEV)
    got = mamba_layer(P.to(DEV), rows, cs, ss, conv_w.to(DEV), conv_b.to(DEV), A_log.to(DEV), dt_bias.to(DEV),
                      D.to(DEV), norm_w.to(DEV), G, N, H, Pd, 1e-5, H * Pd // G, lim)
    torch.cuda.synchronize()
    assert _lib.read_status().get("gdn", 0) == 0
    assert _rel(got.cpu(), want) < 1e-2
    assert _rel(ss.cpu(), ss_r) < 1e-4
    assert torch.equal(cs.cpu(), cs_r.to(torch.bfloat16))


def test_relu2_epilogue():
    x = torch.randn(37, 512, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(384, 512, device=DEV, dtype=torch.bfloat16) * 0.05
    y = ops.gemm(x, w, epi="relu2")
    r = torch.relu(x.float() @ w.float().t()).square()
    assert _rel(y, r) < 1e-2


def test_nemotron_h_engine_graphs_and_oracle():
    hf = {"model_type": "nemotron_h", "vocab_size": 512, "hidden_size": 256, "num_hidden_layers": 6,
          "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64, "mamba_num_heads": 8,
          "mamba_head_dim": 32, "ssm_state_size": 64, "n_groups": 2, "conv_kernel": 4, "intermediate_size": 512,
          "hybrid_override_pattern": "M-M*-M", "layer_norm_epsilon": 1e-5}
    m = DecoderLM(build_config(hf), DEV, torch.bfloat16).init_random(0, std=0.1)
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=16) == eng(False).generate(ps, max_tokens=16)
    p = torch.tensor(ps[1])
    lg = m.forward_dense(p.to(DEV), m.new_cache()).float().cpu()
    mc = m.clone_to("cpu", torch.float32)
    r = mc.forward_dense(p, mc.new_cache())
    assert _rel(lg, r) < 0.05


@pytest.mark.parametrize("C,taps,lens", [(1024, 3, [1, 1, 40, 2, 300]), (2048, 4, [1] * 64)])
def test_short_conv_matches_oracle(C, taps, lens):
    """LFM2 short convolution kernel (and its state roll) against the fp32 oracle."""
    from mlx_swift_lm_b200.ops.gdn import short_conv

    torch.manual_seed(C + taps)
    R = len(lens)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T = cu[-1]
    fresh = [i % 2 for i in range(R)]
    slots = list(range(R))
    P = (torch.randn(T, 3 * C) * 0.5).to(torch.bfloat16)
    w, b = torch.randn(C, taps) * 0.5, torch.randn(C) * 0.1
    cs0 = (torch.randn(R, taps - 1, C) * 0.5).to(torch.bfloat16)
    cs_r = cs0.clone()
    want = ref.short_conv_ref(P.float(), cu, fresh, slots, cs_r, w, b)
    i32 = dict(dtype=torch.int32, device=DEV)
    rows = GdnRows(torch.tensor(cu, **i32), torch.tensor(fresh, **i32), torch.tensor(slots, **i32), cu)
    cs = cs0.to(DEV)
    got = short_conv(P.to(DEV), rows, cs, w.to(DEV), b.to(DEV))
    torch.cuda.synchronize()
    assert _rel(got.cpu(), want) < 1e-2
    assert _rel(cs.cpu(), cs_r.to(torch.bfloat16)) < 1e-2


def test_lfm2_engine_graphs_match_eager():
    hf = {"model_type": "lfm2", "vocab_size": 512, "hidden_size": 256, "num_hidden_layers": 4,
          "num_attention_heads": 4, "num_key_value_heads": 2, "norm_eps": 1e-5, "conv_L_cache": 3,
          "block_ff_dim": 512, "layer_types": ["conv", "full_attention", "conv", "conv"]}
    m = DecoderLM(build_config(hf), DEV, torch.bfloat16).init_random(0, std=0.1)
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=16) == eng(False).generate(ps, max_tokens=16)
