"""ParoQuant pieces on CPU: the pairwise rotation is orthogonal up to the
channel scales, rotated weights compose as y = W (R x), AutoAWQ unpacking."""
import math

import torch

from mlx_swift_lm_b200 import ops
from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight
from mlx_swift_lm_b200.ops.rotation import PairwiseRotation, RotatedWeight, awq_to_quantized, awq_unpack


def _rotation(K=256, krot=3, seed=0, scales=True):
    g = torch.Generator().manual_seed(seed)
    theta = torch.rand(krot, K // 2, generator=g) * math.pi
    pairs = torch.stack([torch.cat([torch.randperm(128, generator=g) for _ in range(K // 128)]) for _ in range(krot)])
    cs = torch.rand(K, generator=g) + 0.5 if scales else None
    return PairwiseRotation(theta, pairs.to(torch.int16), cs), theta, pairs, cs


def test_rotation_is_givens_product():
    r, theta, pairs, cs = _rotation()
    x = torch.randn(5, 256)
    y = r.rotate(x)
    # explicit: scale, then each round's disjoint pair rotations
    t = x * cs
    for k in range(3):
        t = t.clone()
        for gi in range(2):
            for q in range(64):
                i, j = gi * 128 + int(pairs[k, gi * 128 + 2 * q]), gi * 128 + int(pairs[k, gi * 128 + 2 * q + 1])
                c, s = math.cos(theta[k, gi * 64 + q]), math.sin(theta[k, gi * 64 + q])
                a, b = t[:, i].clone(), t[:, j].clone()
                t[:, i], t[:, j] = a * c + b * s, b * c - a * s
    assert torch.allclose(y, t, atol=1e-5)
    r2, *_ = _rotation(scales=False)
    assert torch.allclose(r2.rotate(x).norm(dim=-1), x.norm(dim=-1), atol=1e-4)  # orthogonal


def test_rotated_weight_gemm_and_glu():
    r1, *_ = _rotation(seed=1)
    r2, *_ = _rotation(seed=2)
    w1, w2 = torch.randn(128, 256) * 0.1, torch.randn(64, 256) * 0.1
    rw = RotatedWeight([(r1, w1), (r2, w2)])
    x = torch.randn(7, 256)
    y = ops.gemm(x, rw)
    assert torch.allclose(y, torch.cat([r1.rotate(x) @ w1.t(), r2.rotate(x) @ w2.t()], -1), atol=1e-4)
    glu = RotatedWeight([(r1, w1), (r2, torch.randn(128, 256) * 0.1)], glu=True)
    g = ops.gemm(x, glu, epi="swiglu")
    assert g.shape == (7, 128)


def test_awq_unpack_roundtrip():
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(0, 16, (64, 32), generator=g)
    order = [0, 2, 4, 6, 1, 3, 5, 7]  # AutoAWQ packs nibbles in this order
    c = codes.reshape(64, 4, 8)[..., order]
    packed = torch.zeros(64, 4, dtype=torch.int64)
    for i in range(8):
        packed |= c[..., i].to(torch.int64) << (4 * i)
    packed = packed.to(torch.int32)  # wraps like int32 storage
    assert torch.equal(awq_unpack(packed), codes.to(torch.int32))
    K, N, gs = 128, 32, 64
    qw = torch.randint(0, 16, (K, N), generator=g)
    qz = torch.randint(0, 16, (K // gs, N), generator=g)
    sc = torch.rand(K // gs, N, generator=g) * 0.1

    def pack(a):
        a = a.reshape(a.shape[0], -1, 8)[..., order]
        p = torch.zeros(a.shape[:2], dtype=torch.int64)
        for i in range(8):
            p |= a[..., i].to(torch.int64) << (4 * i)
        return p.to(torch.int32)

    q = awq_to_quantized(pack(qw), pack(qz), sc, gs)
    want = ((qw.float() - qz.float().repeat_interleave(gs, 0)) * sc.repeat_interleave(gs, 0)).t()
    assert isinstance(q, QuantizedWeight) and torch.allclose(q.dequantize(), want, atol=2e-2)


def _awq_pack(a):
    order = [0, 2, 4, 6, 1, 3, 5, 7]
    a = a.reshape(a.shape[0], -1, 8)[..., order]
    p = torch.zeros(a.shape[:2], dtype=torch.int64)
    for i in range(8):
        p |= a[..., i].to(torch.int64) << (4 * i)
    return p.to(torch.int32)


def _awq_quantize(w, gs=64):
    """AutoAWQ tensors of w [N, K] (asymmetric 4-bit per gs inputs)."""
    N, K = w.shape
    g = w.t().reshape(K // gs, gs, N)
    mx, mn = g.amax(1), g.amin(1)
    scale = ((mx - mn) / 15).clamp(min=1e-8)
    zero = torch.round(-mn / scale).clamp(0, 15)
    q = torch.round(g / scale[:, None] + zero[:, None]).clamp(0, 15).reshape(K, N).to(torch.int64)
    return _awq_pack(q), _awq_pack(zero.to(torch.int64)), scale.to(torch.float16)


def test_paroquant_checkpoint_loads_and_matches(tmp_path):
    import json

    from mlx_swift_lm_b200 import DecoderLM
    from mlx_swift_lm_b200.loader.convert import export_tensors, to_hf_config
    from mlx_swift_lm_b200.loader.load import load_model
    from mlx_swift_lm_b200.loader.safetensors import save_safetensors
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(3, std=0.05)
    t = export_tensors(m)
    seed = 10
    for k in list(t):
        if k.endswith("_proj.weight") and t[k].shape[1] % 128 == 0:
            seed += 1
            r, theta, pairs, cs = _rotation(K=t[k].shape[1], krot=2, seed=seed)
            M = r.rotate_ref(torch.eye(t[k].shape[1]))  # R(x) = x @ M
            w_rot = t[k] @ torch.linalg.inv(M).t()  # W_rot R(x) = W x
            qw, qz, sc = _awq_quantize(w_rot)
            base = k[:-len(".weight")]
            del t[k]
            t[base + ".qweight"], t[base + ".qzeros"], t[base + ".scales"] = qw, qz, sc
            t[base + ".theta"], t[base + ".pairs"], t[base + ".channel_scales"] = theta, pairs.to(torch.int16), cs
    d = tmp_path / "paro"
    d.mkdir()
    hf = to_hf_config(m.cfg)
    hf["quantization_config"] = {"quant_method": "paroquant", "bits": 4, "group_size": 64, "krot": 2}
    (d / "config.json").write_text(json.dumps(hf))
    save_safetensors(str(d / "model.safetensors"), t)
    mq, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert isinstance(mq.layers[0].wqkv, RotatedWeight) and len(mq.layers[0].wqkv.parts) == 3
    assert mq.layers[0].wgu.glu
    toks = torch.arange(7, 40)
    a = mq.forward_dense(toks, mq.new_cache())
    md, _ = load_model(str(d), device="cpu", dtype=torch.float32, keep_quantized=False)
    assert torch.allclose(a, md.forward_dense(toks, md.new_cache()), atol=1e-3)  # packed == dequantised path
    b = m.forward_dense(toks, m.new_cache())
    # the original function up to 4-bit error: compare with plain 4-bit quantisation of the same model
    from mlx_swift_lm_b200.models.quantize import quantize_model

    mp = quantize_model(DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(3, std=0.05), bits=4, group_size=64)
    plain = mp.forward_dense(toks, mp.new_cache())
    err, err_plain = ((a - b).norm() / b.norm()).item(), ((plain - b).norm() / b.norm()).item()
    assert err < 1.5 * err_plain, (err, err_plain)
