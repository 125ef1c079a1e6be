"""Checkpoint export (HF / MLX names, optional MLX affine quantisation),
sharded writing and loading back, on tiny models in fp32 on CPU."""
import json
import os

import torch

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.loader.convert import convert, save_model
from mlx_swift_lm_b200.loader.load import load_model
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight


def _model(**over):
    cfg = tiny_qwen3()
    for k, v in over.items():
        setattr(cfg, k, v)
    return DecoderLM(cfg, "cpu", torch.float32).init_random(3, std=0.2)


def _logits(m, toks):
    return m.forward_dense(torch.tensor(toks), m.new_cache())


TOKS = list(range(7, 40))


def test_roundtrip_fp32_sharded(tmp_path):
    m = _model(tie_word_embeddings=False)
    m.lm_head = m.lm_head.clone() * 0.5
    d = str(tmp_path / "ck")
    save_model(m, d, dtype=torch.float32, shard_bytes=2 << 20)
    assert os.path.exists(os.path.join(d, "model.safetensors.index.json"))
    m2, hf = load_model(d, device="cpu", dtype=torch.float32)
    assert hf["model_type"] == "qwen3"
    assert torch.allclose(_logits(m2, TOKS), _logits(m, TOKS), atol=1e-5)


def test_quantized_export_loads_packed(tmp_path):
    m = _model()
    d = str(tmp_path / "q4")
    save_model(m, d, quantize={"bits": 4, "group_size": 64}, dtype=torch.bfloat16)
    cfg = json.load(open(os.path.join(d, "config.json")))
    assert cfg["quantization"] == {"group_size": 64, "bits": 4, "mode": "affine"}
    mq, _ = load_model(d, device="cpu", dtype=torch.float32)
    L = mq.layers[0]
    assert isinstance(L.wqkv, QuantizedWeight) and isinstance(L.wgu, QuantizedWeight)
    assert isinstance(L.wo, QuantizedWeight) and isinstance(L.wd, QuantizedWeight)
    md, _ = load_model(d, device="cpu", dtype=torch.float32, keep_quantized=False)
    a, b = _logits(mq, TOKS), _logits(md, TOKS)
    assert ((a - b).norm() / b.norm()).item() < 2e-2


def test_moe_roundtrip(tmp_path):
    cfg_over = dict(model_type="qwen3_moe", num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
                    norm_topk_prob=True)
    m = _model(**cfg_over)
    d = str(tmp_path / "moe")
    save_model(m, d, dtype=torch.float32)
    m2, _ = load_model(d, device="cpu", dtype=torch.float32)
    assert m2.layers[0].moe
    assert torch.allclose(_logits(m2, TOKS), _logits(m, TOKS), atol=1e-5)


def test_convert_quantizes(tmp_path):
    m = _model()
    src, dst = str(tmp_path / "src"), str(tmp_path / "dst")
    save_model(m, src, dtype=torch.float32)
    with open(os.path.join(src, "tokenizer_config.json"), "w") as f:
        f.write("{}")
    convert(src, dst, {"bits": 8, "group_size": 32})
    assert os.path.exists(os.path.join(dst, "tokenizer_config.json"))
    mq, _ = load_model(dst, device="cpu", dtype=torch.float32)
    assert isinstance(mq.layers[1].wd, QuantizedWeight) and mq.layers[1].wd.bits == 8
    a, ref = _logits(mq, TOKS), _logits(m, TOKS)
    assert ((a - ref).norm() / ref.norm()).item() < 0.05


def test_quantized_moe_experts_load_packed(tmp_path):
    cfg_over = dict(model_type="qwen3_moe", num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
                    norm_topk_prob=True)
    m = _model(**cfg_over)
    d = str(tmp_path / "moeq")
    save_model(m, d, quantize={"bits": 4, "group_size": 64}, dtype=torch.bfloat16)
    mq, _ = load_model(d, device="cpu", dtype=torch.float32)
    L = mq.layers[0]
    assert isinstance(L.experts_gu, QuantizedWeight) and L.experts_gu.num_experts == 8
    assert isinstance(L.experts_d, QuantizedWeight) and L.experts_d.num_experts == 8
    md, _ = load_model(d, device="cpu", dtype=torch.float32, keep_quantized=False)
    a, b = _logits(mq, TOKS), _logits(md, TOKS)
    assert ((a - b).norm() / b.norm()).item() < 2e-2


def test_hf_mxfp4_blocks_pack_exactly():
    from mlx_swift_lm_b200.loader.load import _mxfp4_blocks, _mxfp4_packed

    g = torch.Generator().manual_seed(0)
    E, N, G = 3, 64, 4
    blocks = torch.randint(0, 256, (E, N, G, 16), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = torch.randint(118, 132, (E, N, G), generator=g, dtype=torch.int32).to(torch.uint8)
    q = _mxfp4_packed(blocks, scales)
    assert q.mode == "mxfp4" and q.num_experts == E and q.shape == (E * N, G * 32)
    dense = _mxfp4_blocks(blocks, scales)  # [E, N, K]
    for e in range(E):
        assert torch.equal(q.expert(e).dequantize(), dense[e].to(torch.bfloat16).float())


def _nvfp4_tensors(w):
    from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

    q = QuantizedWeight.quantize_nvfp4(w)
    codes = q.codes_int()
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    g = float(w.abs().max()) / (6.0 * 448.0)
    bs = (q.scales_t.t().float() / g).to(torch.float8_e4m3fn)
    return packed, bs, torch.tensor(g, dtype=torch.float32), q


def test_modelopt_nvfp4_and_fp8_checkpoints(tmp_path):
    from mlx_swift_lm_b200.loader.convert import export_tensors, to_hf_config
    from mlx_swift_lm_b200.loader.safetensors import save_safetensors

    m = _model()
    t = export_tensors(m)
    for k in list(t):
        if k.endswith(("q_proj.weight", "o_proj.weight", "gate_proj.weight", "down_proj.weight")):
            packed, bs, g, _ = _nvfp4_tensors(t[k])
            base = k[:-len(".weight")]
            t[k], t[base + ".weight_scale"], t[base + ".weight_scale_2"] = packed, bs, g
        elif k.endswith(("k_proj.weight", "v_proj.weight", "up_proj.weight")):  # FP8 per-tensor
            s = t[k].abs().max() / 448.0
            base = k[:-len(".weight")]
            t[k], t[base + ".weight_scale"] = (t[k] / s).to(torch.float8_e4m3fn), s.reshape(1)
    d = tmp_path / "mo"
    d.mkdir()
    hf = to_hf_config(m.cfg)
    hf["quantization_config"] = {"quant_method": "modelopt", "quant_algo": "NVFP4"}
    (d / "config.json").write_text(json.dumps(hf))
    save_safetensors(str(d / "model.safetensors"), t)
    mq, _ = load_model(str(d), device="cpu", dtype=torch.float32)
    assert isinstance(mq.layers[0].wo, QuantizedWeight) and mq.layers[0].wo.mode == "nvfp4"
    md, _ = load_model(str(d), device="cpu", dtype=torch.float32, keep_quantized=False)
    a, b = _logits(mq, TOKS), _logits(md, TOKS)
    assert ((a - b).norm() / b.norm()).item() < 1e-3
    ref = _logits(m, TOKS)
    assert ((a - ref).norm() / ref.norm()).item() < 0.5  # fp4 weights: coarse but the same function
