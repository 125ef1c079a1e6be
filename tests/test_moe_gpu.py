"""MoE kernels (router top-k, expert sort, grouped tcgen05 GEMM, combine) vs
plain PyTorch fp32 oracles, and a tiny MoE decoder on the engine."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops import _lib, moe
from mlx_swift_lm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("mode", ["softmax_topk", "topk_softmax"])
@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (64, 128, 8), (300, 128, 4), (17, 256, 8)])
def test_route_topk(mode, T, E, k):
    torch.manual_seed(T + E + k)
    lg = torch.randn(T, E, device=DEV)
    w, ids = moe.route_topk(lg, k, mode, norm_topk=True)
    wr, ir = moe.route_topk(lg.cpu(), k, mode, norm_topk=True)
    assert torch.equal(ids.long().cpu(), ir)
    assert torch.allclose(w.cpu(), wr, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("E,G,TG,k", [(64, 8, 3, 6), (160, 8, 3, 6), (32, 4, 2, 4)])
def test_route_softmax_group_limited(E, G, TG, k):
    """DeepSeek V2 group-limited greedy gate (softmax, groups by best
    probability, no renormalisation, routed scale) against the CPU oracle."""
    torch.manual_seed(E + G)
    lg = torch.randn(200, E, device=DEV) * 2
    w, ids = moe.route_topk(lg, k, "softmax_topk", False, None, G, TG, 16.0)
    wr, ir = moe.route_topk(lg.cpu(), k, "softmax_topk", False, None, G, TG, 16.0)
    assert torch.equal(ids.long().cpu(), ir)
    assert torch.allclose(w.cpu(), wr, atol=1e-5, rtol=1e-4)


def test_route_topk_ties_pick_lower_id():
    lg = torch.zeros(4, 16, device=DEV)
    lg[:, 3] = 1.0
    w, ids = moe.route_topk(lg, 3, "softmax_topk")
    assert ids.cpu().tolist() == [[3, 0, 1]] * 4


@pytest.mark.parametrize("P,E", [(8, 4), (512, 128), (4096, 128), (32768, 256), (100, 1000)])
def test_sort_stable(P, E):
    torch.manual_seed(P)
    ids = torch.randint(0, E, (P,), device=DEV, dtype=torch.int32)
    BN = moe.chunk_rows(P, E)
    mc = (P + BN - 1) // BN + E
    perm = torch.empty(P, dtype=torch.int32, device=DEV)
    pos = torch.empty(P, dtype=torch.int32, device=DEV)
    chunks = torch.empty(3 * mc, dtype=torch.int32, device=DEV)
    nc = torch.empty(1, dtype=torch.int32, device=DEV)
    _lib.check(_lib.lib().b200_moe_sort(ids.data_ptr(), P, E, BN, mc, perm.data_ptr(), pos.data_ptr(),
                                        chunks.data_ptr(), nc.data_ptr(), _lib.stream_ptr(DEV)), "sort")
    torch.cuda.synchronize()
    order = torch.argsort(ids.long().cpu(), stable=True)
    assert torch.equal(perm.long().cpu(), order)
    assert torch.equal(pos.long().cpu()[order], torch.arange(P))
    n = int(nc.item())
    ch = chunks.cpu()[:3 * n].view(n, 3)
    cnt = torch.bincount(ids.long().cpu(), minlength=E)
    assert int(ch[:, 2].sum()) == P
    for e in range(E):
        rows = ch[ch[:, 0] == e]
        assert int(rows[:, 2].sum()) == int(cnt[e])
        assert (rows[:, 2] <= BN).all()


def _moe_ref(h, gu, d, w, idx, epi, gub=None, db=None):
    T, K = h.shape
    out = torch.zeros(T, K)
    for t in range(T):
        for j in range(idx.shape[1]):
            e = int(idx[t, j])
            a = ref.gemm_ref(h[t:t + 1], gu[e], epi, bias=None if gub is None else gub[e])
            y = ref.gemm_ref(a, d[e], bias=None if db is None else db[e])
            out[t] += float(w[t, j]) * y[0].float()
    return out.to(h.dtype)


@pytest.mark.parametrize("epi", ["swiglu", "swiglu_oai"])
@pytest.mark.parametrize("T,E,k,K,F", [(1, 8, 2, 256, 128), (64, 32, 4, 512, 256), (200, 16, 2, 256, 192)])
def test_moe_experts_grouped(epi, T, E, k, K, F):
    torch.manual_seed(T * 3 + E)
    h = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    g = torch.randn(E, F, K, device=DEV, dtype=torch.bfloat16) * 0.05
    u = torch.randn(E, F, K, device=DEV, dtype=torch.bfloat16) * 0.05
    gu = torch.stack([ref.interleave_gate_up(g[e], u[e]) for e in range(E)])
    d = torch.randn(E, K, F, device=DEV, dtype=torch.bfloat16) * 0.05
    gub = torch.randn(E, 2 * F, device=DEV, dtype=torch.bfloat16) * 0.1 if epi == "swiglu_oai" else None
    db = torch.randn(E, K, device=DEV, dtype=torch.bfloat16) * 0.1 if epi == "swiglu_oai" else None
    lg = torch.randn(T, E, device=DEV)
    w, idx = moe.route_topk(lg, k)
    y = moe.moe_experts(h, gu, d, w, idx, epi, gub, db)
    r = _moe_ref(h.cpu(), gu.cpu(), d.cpu(), w.cpu(), idx.cpu(), epi, None if gub is None else gub.cpu(),
                 None if db is None else db.cpu())
    assert _rel(y.cpu(), r) < 2e-2
    y2 = moe.moe_experts(h, gu, d, w, idx, epi, gub, db)
    assert torch.equal(y, y2)  # deterministic


def _moe_model(seed=0):
    cfg = tiny_qwen3()
    cfg.model_type = "qwen3_moe"
    cfg.num_experts = 16
    cfg.num_experts_per_tok = 4
    cfg.moe_intermediate_size = 128
    cfg.norm_topk_prob = True
    return DecoderLM(cfg, DEV, torch.bfloat16).init_random(seed, std=0.2)


def test_moe_model_graph_matches_eager():
    m = _moe_model()
    g = torch.Generator().manual_seed(1)
    ps = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 77)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=16) == eng(False).generate(ps, max_tokens=16)


def test_moe_model_logits_close_to_cpu_oracle():
    m = _moe_model(seed=3)
    p = torch.randint(0, m.cfg.vocab_size, (33,), generator=torch.Generator().manual_seed(4))
    lg = m.forward_dense(p.to(DEV), m.new_cache()).float().cpu()
    mc = m.clone_to("cpu", torch.float32)
    r = mc.forward_dense(p, mc.new_cache())
    # bf16 router logits may flip a near-tied expert choice for a few tokens,
    # so the bound is looser than the dense model's
    assert _rel(lg, r) < 0.15


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("T", [1, 64, 300])
def test_moe_experts_quantized(bits, T):
    from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

    torch.manual_seed(T + bits)
    E, k, K, F = 16, 4, 512, 256
    h = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    gu_f = [ref.interleave_gate_up(torch.randn(F, K) * 0.05, torch.randn(F, K) * 0.05) for _ in range(E)]
    d_f = [torch.randn(K, F) * 0.05 for _ in range(E)]
    gu = QuantizedWeight.stack_experts([QuantizedWeight.quantize(t, bits, 64) for t in gu_f]).to(DEV)
    d = QuantizedWeight.stack_experts([QuantizedWeight.quantize(t, bits, 64) for t in d_f]).to(DEV)
    w, idx = moe.route_topk(torch.randn(T, E, device=DEV), k)
    y = moe.moe_experts(h, gu, d, w, idx)
    gud = torch.stack([gu.expert(e).dequantize() for e in range(E)])
    dd = torch.stack([d.expert(e).dequantize() for e in range(E)])
    r = _moe_ref(h.cpu(), gud.to(torch.bfloat16).cpu(), dd.to(torch.bfloat16).cpu(), w.cpu(), idx.cpu(), "swiglu")
    assert _rel(y.cpu(), r) < 2e-2


def test_quantized_moe_model_graph_matches_eager():
    from mlx_swift_lm_b200.models.quantize import quantize_model

    m = quantize_model(_moe_model(seed=5), bits=4, group_size=64)
    g = torch.Generator().manual_seed(2)
    ps = [torch.randint(0, m.cfg.vocab_size, (n,), generator=g).tolist() for n in (12, 30)]

    def eng(graphs):
        return EngineV2(m, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=4),
                                               max_model_len=256, use_cuda_graphs=graphs, graph_buckets=(1, 2, 4)))

    assert eng(True).generate(ps, max_tokens=12) == eng(False).generate(ps, max_tokens=12)


@pytest.mark.parametrize("T", [1, 64, 300])
def test_moe_experts_mxfp4(T):
    from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

    torch.manual_seed(T + 77)
    E, k, K, F = 16, 4, 512, 256
    h = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    gu_f = [ref.interleave_gate_up(torch.randn(F, K) * 0.05, torch.randn(F, K) * 0.05) for _ in range(E)]
    d_f = [torch.randn(K, F) * 0.05 for _ in range(E)]
    gu = QuantizedWeight.stack_experts([QuantizedWeight.quantize_mxfp4(t) for t in gu_f]).to(DEV)
    d = QuantizedWeight.stack_experts([QuantizedWeight.quantize_mxfp4(t) for t in d_f]).to(DEV)
    gub = torch.randn(E, 2 * F, device=DEV, dtype=torch.bfloat16) * 0.1
    db = torch.randn(E, K, device=DEV, dtype=torch.bfloat16) * 0.1
    w, idx = moe.route_topk(torch.randn(T, E, device=DEV), k, "topk_softmax")
    y = moe.moe_experts(h, gu, d, w, idx, "swiglu_oai", gub, db)
    gud = torch.stack([gu.expert(e).dequantize() for e in range(E)])
    dd = torch.stack([d.expert(e).dequantize() for e in range(E)])
    r = _moe_ref(h.cpu(), gud.to(torch.bfloat16).cpu(), dd.to(torch.bfloat16).cpu(), w.cpu(), idx.cpu(), "swiglu_oai",
                 gub.cpu(), db.cpu())
    assert _rel(y.cpu(), r) < 2e-2


@pytest.mark.parametrize("E,k,n_group,topk_group", [(160, 8, 1, 1), (256, 8, 8, 4), (64, 6, 4, 2)])
def test_sigmoid_group_router_kernel(E, k, n_group, topk_group):
    """GLM-4.5 / DeepSeek-V3 style router on the warp kernel against the CPU re-statement."""
    from mlx_swift_lm_b200.ops import moe as moe_ops

    torch.manual_seed(E + k)
    lg = torch.randn(300, E) * 3
    bias = torch.randn(E) * 0.2
    w_ref, i_ref = moe_ops.route_topk(lg, k, "sigmoid_group", True, bias, n_group, topk_group, 2.5)
    w, i = moe_ops.route_topk(lg.cuda(), k, "sigmoid_group", True, bias.cuda(), n_group, topk_group, 2.5)
    torch.cuda.synchronize()
    assert torch.equal(i.cpu().long(), i_ref)
    assert torch.allclose(w.cpu(), w_ref, atol=1e-5)


def test_e2m1_hardware_pairs():
    """cvt.rn.f16x2.e2m1x2 on every byte: the low nibble lands in the low f16
    of the pair, the high nibble in the high f16, values from the e2m1 table."""
    from mlx_swift_lm_b200.ops import _lib

    out = torch.empty(256, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().b200_e2m1_pairs(out.data_ptr(), _lib.stream_ptr(out.device)), "e2m1_pairs")
    got = out.cpu().view(torch.float16).view(256, 2).float()
    mag = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]

    def val(c):
        return (-1.0 if c & 8 else 1.0) * mag[c & 7]

    want = torch.tensor([[val(b & 15), val(b >> 4)] for b in range(256)])
    assert torch.equal(got, want), (got[:20], want[:20])


@pytest.mark.parametrize("fmt", ["q4", "q8", "mxfp4"])
@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (64, 128, 4), (24, 32, 8)])
def test_persistent_grouped_gemm_equals_per_item(fmt, T, E, k):
    """Decode-sized chunks on persistent CTAs (one per SM, looping over
    (chunk, tile) items, double-buffered accumulators) give the same bits as
    one CTA per item: the same K order and epilogue per output element."""
    from mlx_swift_lm_b200.ops import moe as moe_ops
    from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

    torch.manual_seed(T * 7 + E)
    K, F = 512, 256
    h = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    gu_f = [ref.interleave_gate_up(torch.randn(F, K) * 0.05, torch.randn(F, K) * 0.05) for _ in range(E)]
    d_f = [torch.randn(K, F) * 0.05 for _ in range(E)]
    if fmt == "mxfp4":
        q = QuantizedWeight.quantize_mxfp4
    else:
        bits = 4 if fmt == "q4" else 8

        def q(t):
            return QuantizedWeight.quantize(t, bits, 64)
    gu = QuantizedWeight.stack_experts([q(t) for t in gu_f]).to(DEV)
    d = QuantizedWeight.stack_experts([q(t) for t in d_f]).to(DEV)
    w, idx = moe.route_topk(torch.randn(T, E, device=DEV), k)
    epi = "swiglu_oai" if fmt == "mxfp4" else "swiglu"
    outs = []
    moe_ops.F16_MXFP4[0] = False  # the bf16 dequantising kernels on both launch shapes
    try:
        for pers in (True, False):
            moe_ops.PERSISTENT[0] = pers
            outs.append(moe.moe_experts(h, gu, d, w, idx, epi))
    finally:
        moe_ops.PERSISTENT[0] = False
        moe_ops.F16_MXFP4[0] = True
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert _lib_status_ok()


@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (64, 128, 4), (300, 16, 4)])
def test_mxfp4_f16_path(T, E, k):
    """MXFP4 experts on the f16 path (hardware e2m1 pairs, f16 activations and
    gate/up rows, kind::f16 with f16 operands) against the fp32 reference of
    the dequantised experts, and close to the bf16 path."""
    from mlx_swift_lm_b200.ops import moe as moe_ops
    from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

    torch.manual_seed(T + E)
    K, F = 512, 256
    h = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    gu_f = [ref.interleave_gate_up(torch.randn(F, K) * 0.05, torch.randn(F, K) * 0.05) for _ in range(E)]
    d_f = [torch.randn(K, F) * 0.05 for _ in range(E)]
    gu = QuantizedWeight.stack_experts([QuantizedWeight.quantize_mxfp4(t) for t in gu_f]).to(DEV)
    d = QuantizedWeight.stack_experts([QuantizedWeight.quantize_mxfp4(t) for t in d_f]).to(DEV)
    assert gu.f16_scales_ok() and d.f16_scales_ok()
    gub = torch.randn(E, 2 * F, device=DEV, dtype=torch.bfloat16) * 0.1
    w, idx = moe.route_topk(torch.randn(T, E, device=DEV), k, "topk_softmax")
    y16 = moe.moe_experts(h, gu, d, w, idx, "swiglu_oai", gub)
    moe_ops.PERSISTENT[0] = True  # the persistent launch of the f16 path: the same bits
    try:
        assert torch.equal(moe.moe_experts(h, gu, d, w, idx, "swiglu_oai", gub), y16)
    finally:
        moe_ops.PERSISTENT[0] = False
    moe_ops.F16_MXFP4[0] = False
    try:
        ybf = moe.moe_experts(h, gu, d, w, idx, "swiglu_oai", gub)
    finally:
        moe_ops.F16_MXFP4[0] = True
    gud = torch.stack([gu.expert(e).dequantize() for e in range(E)])
    dd = torch.stack([d.expert(e).dequantize() for e in range(E)])
    r = _moe_ref(h.cpu(), gud.to(torch.bfloat16).cpu(), dd.to(torch.bfloat16).cpu(), w.cpu(), idx.cpu(), "swiglu_oai",
                 gub.cpu())
    assert _rel(y16.cpu(), r) < 2e-2 and _rel(y16.cpu(), ybf.cpu()) < 2e-2
    assert _lib_status_ok()


def _lib_status_ok():
    from mlx_swift_lm_b200.ops import _lib

    return _lib.read_status().get("moe", 0) == 0
