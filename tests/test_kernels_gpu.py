"""sm_100a kernels vs their plain-PyTorch fp32 oracles (ops/reference.py)."""
import math

import pytest
import torch

from mlx_swift_lm_b200 import ops
from mlx_swift_lm_b200.ops import _lib
from mlx_swift_lm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64, 100, 128, 300, 1024])
@pytest.mark.parametrize("N,K", [(256, 256), (384, 1024), (1024, 4096), (4096, 512)])
def test_gemm_bf16(M, N, K):
    torch.manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.05
    y = ops.gemm(x, w)
    r = ref.gemm_ref(x.cpu(), w.cpu())
    assert _rel(y.cpu(), r) < 1e-2
    yf = ops.gemm(x, w, epi="f32")
    assert _rel(yf.cpu(), ref.gemm_ref(x.cpu(), w.cpu(), "f32")) < 1e-3


@pytest.mark.parametrize("epi", ["swiglu", "geglu", "swiglu_oai"])
@pytest.mark.parametrize("M", [3, 64, 200])
def test_gemm_glu_and_bias(epi, M):
    torch.manual_seed(3)
    K, F = 512, 384
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    g = torch.randn(F, K, device=DEV, dtype=torch.bfloat16) * 0.05
    u = torch.randn(F, K, device=DEV, dtype=torch.bfloat16) * 0.05
    w = ref.interleave_gate_up(g, u)
    b = torch.randn(2 * F, device=DEV, dtype=torch.bfloat16) * 0.1
    y = ops.gemm(x, w, epi=epi, bias=b)
    r = ref.gemm_ref(x.cpu(), w.cpu(), epi, bias=b.cpu())
    assert y.shape == (M, F)
    assert _rel(y.cpu(), r) < 1.5e-2


def test_gemm_residual_add():
    torch.manual_seed(4)
    x = torch.randn(40, 256, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(512, 256, device=DEV, dtype=torch.bfloat16) * 0.05
    res = torch.randn(40, 512, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(x, w, epi="add", residual=res)
    assert _rel(y.cpu(), ref.gemm_ref(x.cpu(), w.cpu(), "add", res.cpu())) < 1e-2


def test_gemm_batch_invariance():
    """A row's output does not depend on how many other rows share the GEMM."""
    torch.manual_seed(5)
    K, N = 4096, 6144
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.02
    x = torch.randn(64, K, device=DEV, dtype=torch.bfloat16)
    full = ops.gemm(x, w)
    for m in (1, 5, 16, 33):
        part = ops.gemm(x[:m].contiguous(), w)
        assert torch.equal(part, full[:m]), m


def test_gemm_batch_invariance_across_prefill_sizes():
    """Decode-sized and prefill-sized GEMMs give bit-identical rows (same split order)."""
    torch.manual_seed(15)
    K, N = 4096, 4096
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.02
    x = torch.randn(700, K, device=DEV, dtype=torch.bfloat16)
    big = ops.gemm(x, w)
    for m in (1, 64, 128, 129, 300):
        assert torch.equal(ops.gemm(x[:m].contiguous(), w), big[:m]), m


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
def test_gemm_forced_splits(splits):
    torch.manual_seed(16)
    x = torch.randn(77, 2048, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(640, 2048, device=DEV, dtype=torch.bfloat16) * 0.05
    y = ops.gemm(x, w, splits=splits)
    assert _rel(y.cpu(), ref.gemm_ref(x.cpu(), w.cpu())) < 1e-2


def test_add_rmsnorm():
    torch.manual_seed(6)
    x = torch.randn(17, 4096, device=DEV, dtype=torch.bfloat16)
    d = torch.randn(17, 4096, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(4096, device=DEV, dtype=torch.bfloat16)
    xr, yr = ref.add_rmsnorm_ref(x.cpu(), d.cpu(), w.cpu(), 1e-6)
    y = ops.add_rmsnorm(x, d, w, 1e-6)
    assert torch.equal(x.cpu(), xr)
    assert _rel(y.cpu(), yr) < 5e-3


@pytest.mark.parametrize("H,KVH,D", [(32, 8, 128), (4, 2, 64), (64, 8, 64)])
@pytest.mark.parametrize("fp8", [False, True])
def test_qk_norm_rope_kv(H, KVH, D, fp8):
    from mlx_swift_lm_b200.models.rope import build_rope

    torch.manual_seed(7)
    T, P = 37, 8
    qkv = torch.randn(T, (H + 2 * KVH) * D, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 1000, (T,), device=DEV, dtype=torch.int32)
    slots = torch.randperm(P * 16, device=DEV)[:T].to(torch.int64)
    cs, rot = build_rope(D, 1e6, None, 1024)
    cs = cs.to(DEV)
    qn = torch.randn(D, device=DEV, dtype=torch.bfloat16)
    kn = torch.randn(D, device=DEV, dtype=torch.bfloat16)
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc = torch.zeros(P, KVH, 16, D, device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    ks = torch.rand(KVH, device=DEV) + 0.5 if fp8 else None
    vs = torch.rand(KVH, device=DEV) + 0.5 if fp8 else None
    q = ops.qk_norm_rope_kv(qkv, pos, slots, cs, rot, False, qn, kn, 1e-6, kc, vc, H, KVH, D, ks, vs)
    kc_r = torch.zeros(P, KVH, 16, D, dtype=dt)
    vc_r = torch.zeros_like(kc_r)
    qr, _, _ = ref.qk_norm_rope_kv_ref(qkv.cpu(), pos.cpu(), slots.cpu(), cs.cpu(), rot, False, qn.cpu(), kn.cpu(),
                                       1e-6, kc_r, vc_r, H, KVH, D, None if ks is None else ks.cpu(),
                                       None if vs is None else vs.cpu())
    assert _rel(q.cpu(), qr) < 1e-2
    tol = 0.07 if fp8 else 1e-2
    assert _rel(kc.cpu().float(), kc_r.float()) < tol
    assert _rel(vc.cpu().float(), vc_r.float()) < tol


def _make_paged(B, lens, KVH, D, P, dt=torch.bfloat16):
    maxp = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(P)
    pt = torch.zeros(B, maxp, dtype=torch.int32)
    k = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        pt[b, :n] = perm[k:k + n].to(torch.int32)
        k += n
    kc = (torch.randn(P, KVH, 16, D) * 1.0).to(dt)
    vc = torch.randn(P, KVH, 16, D).to(dt)
    return kc, vc, pt


@pytest.mark.parametrize("H,KVH,D", [(32, 8, 128), (4, 2, 64), (64, 8, 64), (8, 8, 128), (16, 1, 128),
                                     (8, 2, 256)])
@pytest.mark.parametrize("window,sinks", [(0, False), (100, False), (0, True), (128, True)])
def test_paged_decode(H, KVH, D, window, sinks):
    torch.manual_seed(8)
    lens = [1, 15, 16, 17, 255, 256, 257, 700, 1500]
    B = len(lens)
    P = sum((l + 15) // 16 for l in lens) + 5
    kc, vc, pt = _make_paged(B, lens, KVH, D, P)
    q = torch.randn(B, H, D, dtype=torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    sk = torch.randn(H) if sinks else None
    scale = D ** -0.5
    r = ref.paged_decode_ref(q, kc, vc, pt, sl, scale, window, sk)
    y = ops.paged_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), sl.to(DEV), scale, window,
                         None if sk is None else sk.to(DEV))
    assert _rel(y.cpu(), r) < 1e-2


def test_paged_decode_fp8():
    torch.manual_seed(9)
    H, KVH, D = 32, 8, 128
    lens = [33, 400, 1025]
    P = 200
    kc, vc, pt = _make_paged(3, lens, KVH, D, P, torch.float32)
    ks = torch.rand(KVH) + 0.5
    vs = torch.rand(KVH) + 0.5
    kq = (kc / ks[None, :, None, None]).to(torch.float8_e4m3fn)
    vq = (vc / vs[None, :, None, None]).to(torch.float8_e4m3fn)
    q = torch.randn(3, H, D, dtype=torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    r = ref.paged_decode_ref(q, kq, vq, pt, sl, D ** -0.5, k_scale=ks, v_scale=vs)
    y = ops.paged_decode(q.to(DEV), kq.to(DEV), vq.to(DEV), pt.to(DEV), sl.to(DEV), D ** -0.5,
                         k_scale=ks.to(DEV), v_scale=vs.to(DEV))
    assert _rel(y.cpu(), r) < 1e-2


def test_paged_decode_batch_invariance():
    torch.manual_seed(10)
    H, KVH, D = 32, 8, 128
    lens = [300, 1200, 77, 2000]
    P = 300
    kc, vc, pt = _make_paged(4, lens, KVH, D, P)
    q = torch.randn(4, H, D, dtype=torch.bfloat16, device=DEV)
    kc, vc, pt = kc.to(DEV), vc.to(DEV), pt.to(DEV)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    full = ops.paged_decode(q, kc, vc, pt, sl, D ** -0.5)
    for b in range(4):
        one = ops.paged_decode(q[b:b + 1].contiguous(), kc, vc, pt[b:b + 1].contiguous(), sl[b:b + 1], D ** -0.5)
        assert torch.equal(one[0], full[b])


@pytest.mark.parametrize("H,KVH", [(8, 1), (16, 4), (2, 2), (32, 2)])
@pytest.mark.parametrize("window,sinks,softcap,fp8", [(0, False, 0.0, False), (100, True, 0.0, False),
                                                      (0, False, 30.0, False), (0, False, 0.0, True)])
def test_paged_decode_wide(H, KVH, window, sinks, softcap, fp8):
    """Head dim 512 (Gemma 4 global layers): lanes split the head dim."""
    torch.manual_seed(18)
    D = 512
    lens = [1, 16, 17, 256, 257, 900]
    B = len(lens)
    P = sum((l + 15) // 16 for l in lens) + 4
    kc, vc, pt = _make_paged(B, lens, KVH, D, P, torch.float32)
    ks = vs = None
    if fp8:
        ks, vs = torch.rand(KVH) + 0.5, torch.rand(KVH) + 0.5
        kc = (kc / ks[None, :, None, None]).to(torch.float8_e4m3fn)
        vc = (vc / vs[None, :, None, None]).to(torch.float8_e4m3fn)
    else:
        kc, vc = kc.to(torch.bfloat16), vc.to(torch.bfloat16)
    q = torch.randn(B, H, D, dtype=torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    sk = torch.randn(H) if sinks else None
    scale = D ** -0.5
    r = ref.paged_decode_ref(q, kc, vc, pt, sl, scale, window, sk, softcap, ks, vs)
    y = ops.paged_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), sl.to(DEV), scale, window,
                         None if sk is None else sk.to(DEV), softcap, None if ks is None else ks.to(DEV),
                         None if vs is None else vs.to(DEV))
    assert _lib.read_status().get("attn_wide", 0) == 0
    assert _rel(y.cpu(), r) < 1e-2


@pytest.mark.parametrize("window", [0, 40])
def test_paged_prefill_wide(window):
    """Head dim 512 prefill: each chunk token attends as a decode row."""
    torch.manual_seed(19)
    H, KVH, D = 8, 1, 512
    rows = [(0, 37), (100, 64), (16, 1), (250, 300)]
    lens = [h + c for h, c in rows]
    P = sum((l + 15) // 16 for l in lens) + 3
    kc, vc, pt = _make_paged(len(rows), lens, KVH, D, P)
    cu = [0]
    for h, c in rows:
        cu.append(cu[-1] + c)
    q = torch.randn(cu[-1], H, D, dtype=torch.bfloat16)
    cu_t = torch.tensor(cu, dtype=torch.int32)
    p0 = torch.tensor([h for h, _ in rows], dtype=torch.int32)
    r = ref.paged_prefill_ref(q, kc, vc, pt, cu_t, p0, 1.0 / 16, window, None, 0.0)
    y = ops.paged_prefill(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), cu_t.to(DEV), p0.to(DEV), 1.0 / 16,
                          window, cu_q_host=cu)
    assert _rel(y.cpu(), r) < 1e-2


@pytest.mark.parametrize("kernel", ["mma", "simt"])
@pytest.mark.parametrize("H,KVH,D", [(32, 8, 128), (4, 2, 64), (64, 8, 64), (8, 2, 256)])
@pytest.mark.parametrize("window,sinks,softcap", [(0, False, 0.0), (64, True, 0.0), (0, False, 30.0),
                                                  (-1, False, 0.0), (300, False, 0.0)])
def test_paged_prefill(kernel, H, KVH, D, window, sinks, softcap):
    from mlx_swift_lm_b200.ops import attention as att

    if kernel == "simt" and D == 256:
        pytest.skip("the CUDA-core prefill kernel takes D <= 128")
    if kernel == "simt" and window < 0:
        pytest.skip("bidirectional prefill runs on the tensor-core kernels")
    torch.manual_seed(11)
    # rows: (history before the chunk, chunk length)
    rows = [(0, 37), (100, 64), (16, 1), (250, 130), (1000, 200)]
    lens = [h + c for h, c in rows]
    P = sum((l + 15) // 16 for l in lens) + 3
    kc, vc, pt = _make_paged(len(rows), lens, KVH, D, P)
    cu = [0]
    for h, c in rows:
        cu.append(cu[-1] + c)
    T = cu[-1]
    q = torch.randn(T, H, D, dtype=torch.bfloat16)
    cu_t = torch.tensor(cu, dtype=torch.int32)
    p0 = torch.tensor([h for h, _ in rows], dtype=torch.int32)
    sk = torch.randn(H) if sinks else None
    r = ref.paged_prefill_ref(q, kc, vc, pt, cu_t, p0, D ** -0.5, window, sk, softcap)
    att.USE_MMA_PREFILL[0] = kernel != "simt"
    try:
        y = ops.paged_prefill(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), cu_t.to(DEV), p0.to(DEV), D ** -0.5,
                              window, None if sk is None else sk.to(DEV), softcap, cu_q_host=cu)
    finally:
        att.USE_MMA_PREFILL[0] = True
    assert _rel(y.cpu(), r) < 1e-2


def test_argmax_and_sample_match_oracle():
    torch.manual_seed(12)
    B, V = 6, 151936
    logits = torch.randn(B, V) * 3
    a = ops.argmax(logits.to(DEV))
    assert torch.equal(a.cpu(), logits.argmax(-1).to(torch.int32))
    params = [dict(temperature=0.7, top_k=0, top_p=1.0, min_p=0.0, key=11, step=3),
              dict(temperature=1.0, top_k=40, top_p=1.0, min_p=0.0, key=12, step=0),
              dict(temperature=0.9, top_k=0, top_p=0.8, min_p=0.0, key=13, step=9),
              dict(temperature=1.3, top_k=100, top_p=0.5, min_p=0.05, key=14, step=2),
              dict(temperature=0.0, top_k=0, top_p=1.0, min_p=0.0, key=15, step=1),
              dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.2, key=16, step=7)]
    f = lambda k, dt: torch.tensor([p[k] for p in params], dtype=dt, device=DEV)
    keys = torch.tensor([p["key"] for p in params], dtype=torch.int64, device=DEV)
    toks = ops.sample(logits.to(DEV), f("temperature", torch.float32), f("top_k", torch.int32),
                      f("top_p", torch.float32), f("min_p", torch.float32), keys, f("step", torch.int64))
    exp = [ref.sample_ref(logits[b], **{k: v for k, v in params[b].items()}) for b in range(B)]
    assert toks.cpu().tolist() == exp


def test_process_logits_matches_oracle():
    torch.manual_seed(13)
    B, V = 3, 5000
    logits = torch.randn(B, V)
    bias = {5: 2.0, 17: -1.5}
    rep = [3, 3, 9, 100, 5]
    outs = [3, 9, 9, 9, 42]
    exp = torch.stack([ref.process_logits_ref(logits[b], bias, rep, 1.3, outs, 0.4, 0.7) for b in range(B)])
    t = lambda a, dt: torch.tensor(a, dtype=dt, device=DEV)
    lg = logits.to(DEV)
    ops.process_logits(lg, t([[5, 17]] * B, torch.int32), t([[2.0, -1.5]] * B, torch.float32),
                       t([2] * B, torch.int32), t([rep] * B, torch.int32), t([5] * B, torch.int32),
                       t([1.3] * B, torch.float32), t([outs] * B, torch.int32), t([5] * B, torch.int32),
                       t([0.4] * B, torch.float32), t([0.7] * B, torch.float32))
    assert torch.allclose(lg.cpu(), exp, atol=1e-5)


def test_philox_host_matches_numpy():
    import ctypes

    from mlx_swift_lm_b200.ops import _lib
    import numpy as np

    L = _lib.lib()
    idx = np.arange(64)
    host = [L.b200_philox_u32(ctypes.c_uint64(123456789), ctypes.c_uint64(77), int(i)) for i in idx]
    assert host == ref.philox_u32(123456789, 77, idx).tolist()


def test_status_words_clean():
    from mlx_swift_lm_b200.ops import _lib

    st = _lib.read_status()
    assert all(v == 0 for v in st.values()), st


@pytest.mark.parametrize("H,KVH,D", [(32, 8, 128), (64, 8, 64)])
def test_paged_decode_cuda_core_path(H, KVH, D):
    """The CUDA-core partition kernel (fp8 pages use it) stays correct for bf16 too."""
    from mlx_swift_lm_b200.ops import attention as att

    torch.manual_seed(14)
    lens = [5, 300, 1030]
    P = sum((l + 15) // 16 for l in lens) + 2
    kc, vc, pt = _make_paged(3, lens, KVH, D, P)
    q = torch.randn(3, H, D, dtype=torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    r = ref.paged_decode_ref(q, kc, vc, pt, sl, D ** -0.5, 0, None)
    att.USE_MMA_DECODE[0] = False
    try:
        y = ops.paged_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), sl.to(DEV), D ** -0.5)
    finally:
        att.USE_MMA_DECODE[0] = True
    assert _rel(y.cpu(), r) < 1e-2


@pytest.mark.parametrize("V", [151936, 1001])
def test_argmax_nonfinite_flags(V):
    """The greedy pass flags rows holding NaN or +-inf (NaN never wins the
    argmax, so the token alone cannot show it) and leaves finite rows as torch."""
    torch.manual_seed(3)
    x = torch.randn(5, V, device="cuda")
    x[1, 17] = float("nan")
    x[2, V - 1] = float("inf")
    x[3, 0] = -float("inf")
    flags = torch.full((5,), 7, dtype=torch.int32, device="cuda")
    tok = ops.argmax(x, flags=flags)
    torch.cuda.synchronize()
    assert flags.tolist() == [0, 1, 1, 1, 0]
    for r in (0, 3, 4):
        assert tok[r].item() == x[r].argmax().item()
    assert tok[2].item() == V - 1


@pytest.mark.parametrize("M,fp8,norms,bias", [(1, False, True, False), (7, False, True, True), (64, False, True, False),
                                              (64, True, True, False), (300, False, False, True)])
def test_gemm_qkv_rope_matches_unfused(M, fp8, norms, bias):
    """The qkv GEMM with the qk-norm + RoPE + K/V-append epilogue against the
    separate GEMM and qk_norm_rope_kv kernels: same q, same cache contents
    (at most bf16 rounding-order differences in the norm)."""
    from mlx_swift_lm_b200.models.rope import build_rope

    torch.manual_seed(M)
    H, KVH, D, K = 8, 2, 128, 512
    dev = torch.device("cuda")
    N = (H + 2 * KVH) * D
    x = (torch.randn(M, K, device=dev) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device=dev) * 0.1).to(torch.bfloat16) if bias else None
    qn = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16) if norms else None
    kn = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16) if norms else None
    cos_sin, rd = build_rope(D, 1e6, None, 4096)
    cos_sin = cos_sin.to(dev)
    pos = torch.randint(0, 4000, (M,), device=dev, dtype=torch.int32)
    pages = 64
    slots = torch.randperm(pages * 16, device=dev)[:M].to(torch.int64)
    slots[0] = -1  # a padding row writes nothing
    cdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    ks = (torch.rand(KVH, device=dev) + 0.5) if fp8 else None
    vs = (torch.rand(KVH, device=dev) + 0.5) if fp8 else None
    kc1 = torch.zeros(pages, KVH, 16, D, device=dev).to(cdt)
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    qkv = ops.gemm(x, w, bias=b)
    q1 = ops.qk_norm_rope_kv(qkv, pos, slots, cos_sin, rd, False, qn, kn, 1e-6, kc1, vc1, H, KVH, D, ks, vs)
    q2 = ops.gemm_qkv_rope(x, w, b, pos, slots, cos_sin, qn, kn, 1e-6, kc2, vc2, H, KVH, ks, vs)
    torch.cuda.synchronize()
    torch.testing.assert_close(q2.float(), q1.float(), atol=2e-2, rtol=2e-2)
    assert (q2 == q1).float().mean() > 0.95
    for a, c in ((kc2, kc1), (vc2, vc1)):
        torch.testing.assert_close(a.float(), c.float(), atol=6e-2, rtol=6e-2)
    assert _lib.read_status().get("gemm", 0) == 0


@pytest.mark.parametrize("G,window,sinks", [(4, 0, False), (8, 300, True), (1, 0, True)])
def test_decode_fused_merge_matches_separate_merge(G, window, sinks):
    """Tensor-core decode with the split-KV merge fused into the partition
    kernel (last CTA of a row merges, partition order) against the CUDA-core
    kernel + separate merge pass: empty rows give zeros, the arrival counters
    reset themselves (three launches in a row, different batch sizes)."""
    from mlx_swift_lm_b200.ops import attention as att

    torch.manual_seed(G)
    KVH, D, pages = 2, 128, 400
    H = KVH * G
    kc = torch.randn(pages, KVH, 16, D, device="cuda").to(torch.bfloat16)
    vc = torch.randn(pages, KVH, 16, D, device="cuda").to(torch.bfloat16)
    sk = torch.randn(H, device="cuda") if sinks else None
    for B, lens in ((5, [0, 1, 257, 1000, 2047]), (3, [600, 0, 31]), (5, [0, 1, 257, 1000, 2047])):
        q = torch.randn(B, H, D, device="cuda").to(torch.bfloat16)
        pt = torch.randint(0, pages, (B, 128), device="cuda", dtype=torch.int32)
        sl = torch.tensor(lens, device="cuda", dtype=torch.int32)
        att.USE_MMA_DECODE[0] = True
        att.USE_FUSED_MERGE[0] = True
        try:
            fused = ops.paged_decode(q, kc, vc, pt, sl, D ** -0.5, window, sk)
        finally:
            att.USE_FUSED_MERGE[0] = False
        att.USE_MMA_DECODE[0] = False
        try:
            simt = ops.paged_decode(q, kc, vc, pt, sl, D ** -0.5, window, sk)
        finally:
            att.USE_MMA_DECODE[0] = True
        torch.cuda.synchronize()
        for b, n in enumerate(lens):
            if n == 0:
                assert (fused[b] == 0).all()
        torch.testing.assert_close(fused.float(), simt.float(), atol=2e-2, rtol=2e-2)
    assert int(att.merge_counters(q.device, 1)[:B * KVH].abs().sum()) == 0


def test_gemm_row_roles_split_launch():
    """A step of decode rows + prefill rows: the decode rows use the (N, K)
    split, the prefill rows no split; the whole output is written and each
    part equals the GEMM of that part run alone."""
    torch.manual_seed(0)
    x = (torch.randn(300, 512, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(1024, 512, device="cuda") * 0.05).to(torch.bfloat16)
    with ops.row_roles(300, 37):
        y = ops.gemm(x, w)
    y_dec = ops.gemm(x[:37], w)
    y_pf = ops.gemm(x[37:], w, splits=1)
    torch.cuda.synchronize()
    assert y.shape == (300, 1024)
    assert torch.equal(y[:37], y_dec) and torch.equal(y[37:], y_pf)
    torch.testing.assert_close(y.float(), x.float() @ w.float().T, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("N,epi", [(1024, "none"), (384, "none"), (640, "swiglu"), (1280, "f32"), (768, "add"),
                                   (512, "gelu")])
def test_gemm_two_tile_unsplit(N, epi):
    """Unsplit GEMMs with >128 rows run 256 x 256 tiles (two weight tiles and
    two accumulators per CTA); N not a multiple of 256 leaves a half-used last
    tile. Checked against the fp32 oracle and the split-K path."""
    torch.manual_seed(N)
    M, K = 300, 1024
    x = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda") * 0.1).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda").to(torch.bfloat16) if epi == "add" else None
    y1 = ops.gemm(x, w, epi=epi, residual=r, bias=b, splits=1)
    y4 = ops.gemm(x, w, epi=epi, residual=r, bias=b, splits=4)
    want = ref.gemm_ref(x.float(), w.float(), epi, r.float() if r is not None else None, bias=b.float())
    torch.cuda.synchronize()
    torch.testing.assert_close(y1.float(), want.float(), atol=5e-2, rtol=5e-2)
    torch.testing.assert_close(y1.float(), y4.float(), atol=5e-2, rtol=5e-2)


def test_gemm_qkv_rope_two_tile():
    """The fused qkv epilogue on the 256 x 256 tile path (unsplit, >128 rows)."""
    from mlx_swift_lm_b200.models.rope import build_rope

    torch.manual_seed(9)
    H, KVH, D, K, M = 6, 1, 128, 512, 260  # 8 heads: the last CTA's second tile is a value head
    dev = torch.device("cuda")
    N = (H + 2 * KVH) * D
    x = (torch.randn(M, K, device=dev) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
    cos_sin, rd = build_rope(D, 1e6, None, 4096)
    cos_sin = cos_sin.to(dev)
    pos = torch.randint(0, 4000, (M,), device=dev, dtype=torch.int32)
    slots = torch.randperm(64 * 16, device=dev)[:M].to(torch.int64)
    kc1 = torch.zeros(64, KVH, 16, D, device=dev, dtype=torch.bfloat16)
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    qkv = ops.gemm(x, w, splits=1)
    q1 = ops.qk_norm_rope_kv(qkv, pos, slots, cos_sin, rd, False, qn, kn, 1e-6, kc1, vc1, H, KVH, D)
    q2 = ops.gemm_qkv_rope(x, w, None, pos, slots, cos_sin, qn, kn, 1e-6, kc2, vc2, H, KVH, splits=1)
    torch.cuda.synchronize()
    torch.testing.assert_close(q2.float(), q1.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(kc2.float(), kc1.float(), atol=6e-2, rtol=6e-2)
    assert torch.equal(vc2, vc1)


def test_xielu_kernel_matches_oracle():
    torch.manual_seed(2)
    x = (torch.randn(37, 1000) * 3).to(torch.bfloat16)
    p = torch.tensor([0.3, -0.2, 0.5, -1e-6])
    want = ref.xielu_ref(x, p).float()
    y = ops.xielu(x.to("cuda").contiguous(), p.to("cuda"))
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float().cpu(), want, atol=3e-2, rtol=2e-2)
