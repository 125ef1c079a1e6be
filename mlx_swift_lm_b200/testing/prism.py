"""Writer of synthetic Prism Hadamard artifacts (schema 2) from a dense
Qwen 3.5-style hybrid decoder, for tests and benchmarks without a download.

Every declared module stores its weight W as the 2-bit affine group-128
quantisation of the forward-transformed rows H(s * w) / sqrt(b) (the layout
the transformed linear ``((x * s) H) W_q^T`` expects); the embedding is
stored the same way and read back through the inverse transform. The
returned dict holds the dense tensors the artifact is equivalent to (each
module's dequantised rows, rounded once to bf16 as the dequantising GEMM
does, inverse-transformed), so a dense model built from them is the oracle
of the packed one. Scales and biases are float16 values that bf16 represents
exactly (the packed records hold bf16 scales).
"""
from __future__ import annotations

import json
import os

import torch

from ..loader.convert import export_tensors, to_hf_config, write_shards
from ..loader.prism import MODEL_TYPE
from ..ops import quant
from ..ops.rotation import HadamardTransform

GROUP = 128
BITS = 2


def _qwen35_names(model, t: dict) -> dict:
    """Qwen3-Next exported names -> Qwen 3.5 ones (separate in_proj_qkv / z / b / a)."""
    Hk, Dk, Hv, Dv = model.cfg.gdn_dims
    kd, vd = Hk * Dk, Hv * Dv
    for i, L in enumerate(model.layers):
        if not L.linear:
            continue
        la = f"model.layers.{i}.linear_attn."
        w = L.wqkv.float() if isinstance(L.wqkv, torch.Tensor) else L.wqkv.dequantize(torch.float32)
        del t[la + "in_proj_qkvz.weight"], t[la + "in_proj_ba.weight"]
        t[la + "in_proj_qkv.weight"] = w[:2 * kd + vd]
        t[la + "in_proj_z.weight"] = w[2 * kd + vd:2 * kd + 2 * vd]
        t[la + "in_proj_b.weight"] = w[2 * kd + 2 * vd:2 * kd + 2 * vd + Hv]
        t[la + "in_proj_a.weight"] = w[2 * kd + 2 * vd + Hv:]
    return t


def write_prism_checkpoint(model, path: str, block: int = 512, seed: int = 0) -> dict:
    """Write config.json, hadamard.json and the safetensors shards of `model`
    as a Prism artifact; returns the equivalent dense tensors (same names)."""
    cfg = model.cfg
    t = _qwen35_names(model, export_tensors(model))
    if "lm_head.weight" not in t:
        t["lm_head.weight"] = t["model.embed_tokens.weight"].clone()
    g = torch.Generator().manual_seed(seed)
    signs: dict[int, torch.Tensor] = {}

    def transform(width):
        if width not in signs:
            signs[width] = (torch.randint(0, 2, (width,), generator=g) * 2 - 1).float()
        return HadamardTransform(block, signs[width])

    def declared(name, w):
        if name == "model.embed_tokens.weight":
            return True
        return (w.dim() == 2 and name.endswith(".weight") and "norm" not in name and "conv1d" not in name
                and w.shape[1] % block == 0 and w.shape[1] % GROUP == 0)

    out, dense, modules, fwd, inv = {}, {}, [], [], []
    for name, w in t.items():
        key = "language_model." + name
        if not declared(name, w):
            v = w.float() if w.is_floating_point() else w
            out[key] = dense[key] = v
            continue
        tr = transform(w.shape[1])
        packed, s, b = quant.affine_quantize(tr.rotate(w.float()), GROUP, BITS)
        # float16 scales / biases that bf16 holds exactly (the packed records
        # keep bf16), and rows rounded once to bf16 (the tensor-core operand)
        s, b = s.bfloat16().half(), b.bfloat16().half()
        rows = quant.dequantize(packed, s, b, "affine", GROUP, BITS, torch.float32)
        emb = name == "model.embed_tokens.weight"
        dense[key] = tr.inverse(rows if emb else rows.bfloat16().float())  # the table is dequantised in fp32
        base = key[:-len(".weight")]
        out[key], out[base + ".scales"], out[base + ".biases"] = packed, s, b
        out[base + ".signs"] = signs[w.shape[1]].clone()
        modules.append({"path": base[len("language_model."):], "block": block, "embedding": emb, "dtype": "float16"})
        (inv if emb else fwd).append(key)
    text = to_hf_config(cfg)
    text["model_type"] = "qwen3_5_text"
    text["tie_word_embeddings"] = False  # the head is its own module
    text.pop("quantization", None)
    hf = {"schema_version": 2, "model_type": MODEL_TYPE, "base_model_type": "qwen3_5",
          "gdn_activation_layout": "grouped", "tensor_namespace": "mlx-vlm-qwen3_5", "hadamard_config": "hadamard.json",
          "components": {"text": True, "vision": False, "mtp": False},
          "quantization": {"bits": BITS, "group_size": GROUP, "mode": "affine"}, "text_config": text,
          "modules": modules}
    widths = sorted(signs)
    meta = {"prism.hadamard.version": 1, "prism.hadamard.block_size": block,
            "prism.hadamard.transform": "normalized-sylvester-walsh-hadamard",
            "prism.hadamard.axis": "input-last-dimension", "prism.hadamard.sign_mode": "explicit",
            "prism.hadamard.weight_names": fwd, "prism.hadamard.inverse_weight_names": inv,
            "prism.hadamard.sign_widths": widths,
            "prism.hadamard.sign_values": [float(v) for w in widths for v in signs[w].tolist()],
            "prism.hadamard.gdn_v_grouped": True}
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
    with open(os.path.join(path, "hadamard.json"), "w") as f:
        json.dump(meta, f)
    write_shards(out, path)
    return dense
