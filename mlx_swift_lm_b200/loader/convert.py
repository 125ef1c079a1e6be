"""Model conversion: write a :class:`DecoderLM` (or a converted checkpoint) as
a Hugging Face / MLX directory, optionally quantising the linear layers in
MLX's affine format.

Parity: ModelConversion (MLXLMCommon/ModelConversion.swift,
MLXLLM/ModelConversion.swift): load, optionally quantise
(``quantization {group_size, bits, mode}`` in config.json with ``weight`` /
``scales`` / ``biases`` per quantised linear), save shards plus config.

The model's fused layouts are undone on export: q|k|v is split back into
q_proj / k_proj / v_proj and the 64-row interleaved gate/up into gate_proj /
up_proj, so any loader that reads HF names (including this one) accepts the
result. Tensor-parallel shards cannot be exported (world 1 only).

CLI (mlx_lm.convert style):
    python -m mlx_swift_lm_b200.loader.convert --src DIR --dst DIR [--q-bits 4 --q-group-size 64] [--dtype bf16]
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..models.families import FAMILIES
from ..ops import quant
from ..ops.qlinear import QuantizedWeight
from ..ops.reference import deinterleave_gate_up
from .safetensors import save_safetensors

# names of the linears that quantisation covers (MLX quantises every Linear
# whose input size divides the group size; embeddings too)
_QUANTISABLE = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "lm_head",
                "embed_tokens")


def to_hf_config(cfg, quantization: dict | None = None) -> dict:
    d = {"model_type": cfg.model_type, "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size,
         "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
         "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
         "intermediate_size": cfg.intermediate_size, "rms_norm_eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta,
         "max_position_embeddings": cfg.max_position_embeddings, "tie_word_embeddings": cfg.tie_word_embeddings,
         "attention_bias": cfg.attention_bias, "mlp_bias": cfg.mlp_bias, "hidden_act": "silu"}
    if cfg.rope_scaling:
        d["rope_scaling"] = cfg.rope_scaling
    if cfg.partial_rotary_factor != 1.0:
        d["partial_rotary_factor"] = cfg.partial_rotary_factor
    if cfg.num_experts:
        d.update(num_experts=cfg.num_experts, num_experts_per_tok=cfg.num_experts_per_tok,
                 moe_intermediate_size=cfg.moe_intermediate_size, norm_topk_prob=cfg.norm_topk_prob)
        if cfg.moe_layers is not None:
            d["mlp_only_layers"] = [i for i, x in enumerate(cfg.moe_layers) if not x]
        if cfg.shared_expert_intermediate_size:
            d["shared_expert_intermediate_size"] = cfg.shared_expert_intermediate_size
        if cfg.router_mode == "sigmoid_group":  # GLM-4.5-style keys
            first = next((i for i, x in enumerate(cfg.moe_layers or []) if x), 0)
            d.update(n_routed_experts=cfg.num_experts, first_k_dense_replace=first, n_group=cfg.router_n_group,
                     topk_group=cfg.router_topk_group, routed_scaling_factor=cfg.routed_scaling_factor,
                     n_shared_experts=cfg.shared_expert_intermediate_size // max(cfg.moe_intermediate_size, 1),
                     use_qk_norm=cfg.qk_norm, scoring_func="sigmoid")
    if cfg.extra.get("mla"):  # DeepSeek-style keys: latent attention dims and the router
        e = cfg.extra
        first = next((i for i, x in enumerate(cfg.moe_layers or []) if x), cfg.num_layers)
        d.update(q_lora_rank=e["mla_q_lora"] or None, kv_lora_rank=e["mla_kv_lora"],
                 qk_nope_head_dim=e["mla_qk_nope"], qk_rope_head_dim=e["mla_qk_rope"], v_head_dim=e["mla_v"],
                 n_routed_experts=cfg.num_experts, first_k_dense_replace=first, n_group=cfg.router_n_group,
                 topk_group=cfg.router_topk_group, routed_scaling_factor=cfg.routed_scaling_factor,
                 n_shared_experts=cfg.shared_expert_intermediate_size // max(cfg.moe_intermediate_size, 1),
                 norm_topk_prob=cfg.norm_topk_prob,
                 scoring_func="sigmoid" if cfg.router_mode == "sigmoid_group" else "softmax",
                 topk_method="group_limited_greedy" if cfg.router_n_group > 1 else "greedy")
        d.pop("num_key_value_heads")
        d.pop("head_dim")
        d.pop("partial_rotary_factor", None)
    if cfg.layer_types:
        d.update(layer_types=list(cfg.layer_types), attn_output_gate=cfg.attn_output_gate,
                 linear_num_key_heads=cfg.linear_num_key_heads, linear_num_value_heads=cfg.linear_num_value_heads,
                 linear_key_head_dim=cfg.linear_key_head_dim, linear_value_head_dim=cfg.linear_value_head_dim,
                 linear_conv_kernel_dim=cfg.linear_conv_kernel_dim)
    if quantization:
        d["quantization"] = dict(quantization)
    return d


def _dense(t) -> torch.Tensor:
    if isinstance(t, QuantizedWeight):
        return t.dequantize(torch.float32)
    return t.detach().float().cpu()


def _export_linear_attn(out: dict, la: str, L, cfg):
    """Gated DeltaNet weights under Qwen3-Next names (in_proj_qkvz / in_proj_ba
    packed per key head) with conv taps as [C, K, 1] (the MLX layout, whose
    layer norms already hold 1 + w)."""
    Hk, Dk, Hv, Dv = cfg.gdn_dims
    vpk = Hv // Hk
    w = _dense(L.wqkv)
    kd, vd = Hk * Dk, Hv * Dv
    q, k, v, z = w[:kd], w[kd:2 * kd], w[2 * kd:2 * kd + vd], w[2 * kd + vd:2 * kd + 2 * vd]
    b, a = w[2 * kd + 2 * vd:2 * kd + 2 * vd + Hv], w[2 * kd + 2 * vd + Hv:]
    H = w.shape[1]
    qkvz = torch.cat([q.view(Hk, Dk, H), k.view(Hk, Dk, H), v.view(Hk, vpk * Dv, H), z.view(Hk, vpk * Dv, H)], 1)
    out[la + "in_proj_qkvz.weight"] = qkvz.reshape(-1, H)
    out[la + "in_proj_ba.weight"] = torch.cat([b.view(Hk, vpk, H), a.view(Hk, vpk, H)], 1).reshape(-1, H)
    out[la + "conv1d.weight"] = _dense(L.conv_w)[:, :, None]
    out[la + "A_log"] = _dense(L.A_log)
    out[la + "dt_bias"] = _dense(L.dt_bias)
    out[la + "norm.weight"] = _dense(L.gdn_norm)
    out[la + "out_proj.weight"] = _dense(L.wo)


def export_tensors(model) -> dict[str, torch.Tensor]:
    """HF-named fp32 tensors of a world-1 model."""
    if model.tp.world != 1:
        raise ValueError("export needs the unsharded model (tensor-parallel world 1)")
    cfg = model.cfg
    gemma = bool(FAMILIES.get(cfg.model_type, {}).get("gemma"))
    off = 1.0 if gemma else 0.0  # the loader folds Gemma's (1 + w) into the stored norm weights
    out = {"model.embed_tokens.weight": _dense(model.embed), "model.norm.weight": _dense(model.norm) - off}
    if model.lm_head is not model.embed and not cfg.tie_word_embeddings:
        out["lm_head.weight"] = _dense(model.lm_head)
    qn, kn = model.H * model.D, model.KVH * model.D
    for i, L in enumerate(model.layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = _dense(L.ln1) - off
        if L.post_attn_norm is not None:
            out[p + "post_attention_layernorm.weight"] = _dense(L.post_attn_norm) - off
            out[p + "pre_feedforward_layernorm.weight"] = _dense(L.ln2) - off
            out[p + "post_feedforward_layernorm.weight"] = _dense(L.post_ffn_norm) - off
        else:
            out[p + "post_attention_layernorm.weight"] = _dense(L.ln2) - off
        a = p + "self_attn."
        w = _dense(L.wqkv) if L.wqkv is not None else None
        if L.mla_kv_a is not None:
            if L.mla_q_a is not None:
                out[a + "q_a_proj.weight"] = _dense(L.mla_q_a)
                out[a + "q_a_layernorm.weight"] = _dense(L.mla_q_a_norm)
                out[a + "q_b_proj.weight"] = _dense(L.mla_q_b)
            else:
                out[a + "q_proj.weight"] = _dense(L.mla_q_b)
            out[a + "kv_a_proj_with_mqa.weight"] = _dense(L.mla_kv_a)
            out[a + "kv_a_layernorm.weight"] = _dense(L.mla_kv_a_norm)
            out[a + "kv_b_proj.weight"] = _dense(L.mla_kv_b)
        elif L.linear:
            _export_linear_attn(out, p + "linear_attn.", L, cfg)
        elif cfg.attn_output_gate:  # q_proj rows per head [q | gate]
            H, D = model.H, model.D
            q, gt = w[:qn].view(H, D, -1), w[qn + 2 * kn:].view(H, D, -1)
            out[a + "q_proj.weight"] = torch.cat([q, gt], 1).reshape(2 * qn, -1)
            out[a + "k_proj.weight"], out[a + "v_proj.weight"] = w[qn:qn + kn], w[qn + kn:qn + 2 * kn]
        else:
            out[a + "q_proj.weight"], out[a + "k_proj.weight"], out[a + "v_proj.weight"] = (
                w[:qn], w[qn:qn + kn], w[qn + kn:])
        if L.linear:
            pass
        elif L.bqkv is not None:
            b = _dense(L.bqkv)
            out[a + "q_proj.bias"], out[a + "k_proj.bias"], out[a + "v_proj.bias"] = b[:qn], b[qn:qn + kn], b[qn + kn:]
        if L.q_norm is not None:
            out[a + "q_norm.weight"] = _dense(L.q_norm) - off
            out[a + "k_norm.weight"] = _dense(L.k_norm) - off
        if not L.linear:
            out[a + "o_proj.weight"] = _dense(L.wo)
        if L.bo is not None:
            out[a + "o_proj.bias"] = _dense(L.bo)
        if L.sinks is not None:
            out[a + "sinks"] = _dense(L.sinks)
        mp = p + "mlp."
        if L.moe:
            if cfg.model_type == "gpt_oss":
                raise ValueError("export of gpt-oss expert layouts is not supported")
            out[mp + "gate.weight"] = _dense(L.router)
            if L.router_corr is not None:
                out[mp + "gate.e_score_correction_bias"] = _dense(L.router_corr)
            E = L.experts_gu.num_experts if isinstance(L.experts_gu, QuantizedWeight) else L.experts_gu.shape[0]
            for e in range(E):
                ge = L.experts_gu.expert(e) if isinstance(L.experts_gu, QuantizedWeight) else L.experts_gu[e]
                de = L.experts_d.expert(e) if isinstance(L.experts_d, QuantizedWeight) else L.experts_d[e]
                g, u = deinterleave_gate_up(_dense(ge))
                out[f"{mp}experts.{e}.gate_proj.weight"] = g
                out[f"{mp}experts.{e}.up_proj.weight"] = u
                out[f"{mp}experts.{e}.down_proj.weight"] = _dense(de)
            if L.shared_gu is not None:
                g, u = deinterleave_gate_up(_dense(L.shared_gu))
                sp = mp + ("shared_experts." if cfg.router_mode == "sigmoid_group" or cfg.extra.get("mla")
                       else "shared_expert.")
                out[sp + "gate_proj.weight"] = g
                out[sp + "up_proj.weight"] = u
                out[sp + "down_proj.weight"] = _dense(L.shared_d)
                if L.shared_gate is not None:
                    out[mp + "shared_expert_gate.weight"] = _dense(L.shared_gate)
        else:
            g, u = deinterleave_gate_up(_dense(L.wgu))
            out[mp + "gate_proj.weight"], out[mp + "up_proj.weight"] = g, u
            out[mp + "down_proj.weight"] = _dense(L.wd)
            if L.bgu is not None:
                gb, ub = deinterleave_gate_up(_dense(L.bgu)[:, None])
                out[mp + "gate_proj.bias"], out[mp + "up_proj.bias"] = gb[:, 0], ub[:, 0]
            if L.bd is not None:
                out[mp + "down_proj.bias"] = _dense(L.bd)
    return out


def quantize_tensors(tensors: dict, bits: int = 4, group_size: int = 64, dtype=torch.bfloat16) -> dict:
    """MLX affine quantisation of every quantisable 2-D weight whose input
    size is a multiple of the group size; scales / biases in `dtype`."""
    out = {}
    for name, t in tensors.items():
        base = name[:-len(".weight")] if name.endswith(".weight") else None
        leaf = base.rsplit(".", 1)[-1] if base else ""
        if base and t.dim() == 2 and leaf in _QUANTISABLE and t.shape[1] % group_size == 0:
            packed, s, b = quant.affine_quantize(t.float(), group_size, bits)
            out[name] = packed
            out[base + ".scales"] = s.to(dtype)
            out[base + ".biases"] = b.to(dtype)
        else:
            out[name] = t
    return out


def export_vision_tensors(model) -> dict:
    """HF names (``visual.*``) of a Qwen2-VL vision tower."""
    v = model.vision
    out = {"visual.patch_embed.proj.weight": v.patch_w.detach().float().cpu().reshape(
        v.cfg.embed_dim, v.cfg.in_chans, v.cfg.temporal_patch_size, v.cfg.patch_size, v.cfg.patch_size)}
    names = {"norm1_w": "norm1.weight", "norm1_b": "norm1.bias", "norm2_w": "norm2.weight", "norm2_b": "norm2.bias",
             "qkv_w": "attn.qkv.weight", "qkv_b": "attn.qkv.bias", "proj_w": "attn.proj.weight",
             "proj_b": "attn.proj.bias", "fc1_w": "mlp.fc1.weight", "fc1_b": "mlp.fc1.bias", "fc2_w": "mlp.fc2.weight",
             "fc2_b": "mlp.fc2.bias"}
    for i, b in enumerate(v.blocks):
        for s, n in names.items():
            out[f"visual.blocks.{i}.{n}"] = getattr(b, s).detach().float().cpu()
    for s, n in (("ln_q_w", "ln_q.weight"), ("ln_q_b", "ln_q.bias"), ("m1_w", "mlp.0.weight"), ("m1_b", "mlp.0.bias"),
                 ("m2_w", "mlp.2.weight"), ("m2_b", "mlp.2.bias")):
        out[f"visual.merger.{n}"] = getattr(v, s).detach().float().cpu()
    return out


def save_model(model, path: str, quantize: dict | None = None, dtype=torch.bfloat16, shard_bytes: int = 5 << 30):
    """Write config.json + model(-NNNNN-of-NNNNN).safetensors (+ index) for `model`."""
    os.makedirs(path, exist_ok=True)
    tensors = export_tensors(model)
    qcfg = None
    if quantize:
        qcfg = {"group_size": int(quantize.get("group_size", 64)), "bits": int(quantize.get("bits", 4)),
                "mode": "affine"}
        tensors = quantize_tensors(tensors, qcfg["bits"], qcfg["group_size"], dtype)
    hfc = to_hf_config(model.cfg, qcfg)
    if getattr(model, "vision", None) is not None:  # Qwen2-VL: the tower stays unquantised
        tensors.update(export_vision_tensors(model))
        vc = model.vision.cfg
        hfc.update(vision_config={"depth": vc.depth, "embed_dim": vc.embed_dim, "num_heads": vc.num_heads,
                                  "mlp_ratio": vc.mlp_ratio, "patch_size": vc.patch_size,
                                  "temporal_patch_size": vc.temporal_patch_size,
                                  "spatial_merge_size": vc.spatial_merge_size, "in_chans": vc.in_chans,
                                  "hidden_size": vc.hidden_size},
                   image_token_id=model.image_token_id, video_token_id=model.video_token_id,
                   rope_scaling={"type": "mrope", "mrope_section": list(model.mrope_section)})
    tensors = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in tensors.items()}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hfc, f, indent=2)
    write_shards(tensors, path, shard_bytes)


def write_shards(tensors: dict, path: str, shard_bytes: int = 5 << 30):
    shards, cur, size = [], {}, 0
    for k in sorted(tensors):
        t = tensors[k]
        nb = t.numel() * t.element_size()
        if cur and size + nb > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t
        size += nb
    if cur:
        shards.append(cur)
    if len(shards) == 1:
        save_safetensors(os.path.join(path, "model.safetensors"), shards[0], {"format": "pt"})
        return
    wmap = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_safetensors(os.path.join(path, fn), sh, {"format": "pt"})
        wmap.update({k: fn for k in sh})
    total = sum(t.numel() * t.element_size() for t in tensors.values())
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": wmap}, f, indent=2)


def convert(src: str, dst: str, quantize: dict | None = None, dtype=torch.bfloat16):
    """Load a checkpoint directory (dequantising it) and write it to `dst`."""
    from .load import load_model

    model, hf = load_model(src, device="cpu", dtype=torch.float32, keep_quantized=False)
    save_model(model, dst, quantize, dtype)
    for extra in ("tokenizer.json", "tokenizer_config.json", "generation_config.json", "special_tokens_map.json",
                  "chat_template.jinja"):
        sp = os.path.join(src, extra)
        if os.path.exists(sp):
            with open(sp, "rb") as fi, open(os.path.join(dst, extra), "wb") as fo:
                fo.write(fi.read())


def main(argv=None):
    ap = argparse.ArgumentParser(description="convert / quantise a checkpoint directory")
    ap.add_argument("--src", required=True)
    ap.add_argument("--dst", required=True)
    ap.add_argument("--q-bits", type=int, default=0)
    ap.add_argument("--q-group-size", type=int, default=64)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp16", "fp32"])
    a = ap.parse_args(argv)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[a.dtype]
    q = {"bits": a.q_bits, "group_size": a.q_group_size} if a.q_bits else None
    convert(a.src, a.dst, q, dt)


if __name__ == "__main__":
    main()
