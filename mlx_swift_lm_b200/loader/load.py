"""Checkpoint loading: HF / MLX directories -> :class:`DecoderLM`.

Parity: ``loadModelContainer`` (MLXLMCommon/ModelFactory.swift:310) resolves a
directory, reads ``config.json``, dispatches on ``model_type`` and runs
``loadWeights`` (Load.swift:522): read every shard, per-model ``sanitize``
(drop ``lm_head`` for tied models, Qwen3.swift:200-207), quantized modules
from ``scales``/``biases`` (``applyCheckpoint`` :651), convert to bf16 (:733).

Here the per-family sanitize step is the name mapping below; projections are
fused at load (q|k|v into one weight, gate/up interleaved in 64-row blocks
for the SwiGLU GEMM epilogue) and sliced for tensor parallelism.
MLX affine / MXFP4 / NVFP4 / MXFP8 weights are kept in their packed layout
(:class:`QuantizedWeight`) when a dequantising kernel serves them, and are
dequantised to bf16 otherwise.
"""
from __future__ import annotations

import json
import math
import os

import torch

from ..models.config import DecoderConfig
from ..models.decoder import DecoderLM, LayerWeights, TensorParallel
from ..models.families import build_config
from ..ops import quant
from ..ops.qlinear import CARRIED_BITS, SUPPORTED_GROUPS, QuantizedWeight
from ..ops.reference import interleave_gate_up as _interleave_dense
from . import prism
from .safetensors import load_safetensors


def _same_format(parts) -> bool:
    p0 = parts[0]
    return all(isinstance(p, QuantizedWeight) and (p.bits, p.gs, p.mode) == (p0.bits, p0.gs, p0.mode) for p in parts)


def _dense(t):
    return t.dequantize(torch.float32) if isinstance(t, QuantizedWeight) else t


def _rotated(parts) -> bool:
    from ..ops.rotation import RotatedWeight

    return any(isinstance(p, RotatedWeight) for p in parts)


def _as_rotated(w):
    from ..ops.rotation import RotatedWeight

    return w if isinstance(w, RotatedWeight) else RotatedWeight([(None, w)])


def interleave_gate_up(g, u):
    """Gate / up rows in 64-row interleaved blocks; packed when both share a
    quantised format, else dense (mixed-format checkpoints); rotated (ParoQuant)
    gate / up keep their own rotations as a GLU pair."""
    if _rotated([g, u]):
        from ..ops.rotation import RotatedWeight

        return RotatedWeight(_as_rotated(g).parts + _as_rotated(u).parts, glu=True)
    if _same_format([g, u]):
        return QuantizedWeight.interleave_gate_up(g, u)
    return _interleave_dense(_dense(g), _dense(u))


def _cat_rows(parts):
    if _rotated(parts):
        from ..ops.rotation import RotatedWeight

        return RotatedWeight([pr for p in parts for pr in _as_rotated(p).parts])
    if _same_format(parts):
        return QuantizedWeight.cat_rows(parts)
    return torch.cat([_dense(p) for p in parts], 0)


class CheckpointView:
    """Name lookup over a flat tensor dict with prefix detection and MLX-quantized
    linear dequantisation."""

    def __init__(self, tensors: dict, qcfg: dict | None, dtype, keep_quantized: bool = False, hadamard=None):
        self.t = tensors
        self.q = qcfg or {}
        self.dtype = dtype
        self.keep_quantized = keep_quantized
        self.hadamard = hadamard  # Prism Hadamard metadata (loader.prism.HadamardMetadata)
        keys = list(tensors)
        self.prefix = ""
        for pre in ("model.language_model.", "language_model.model.", "model.text_model.", "text_model.", "model.",
                    "transformer.", "encoder.", "backbone.", ""):
            if any(k.startswith(pre + "layers.0.") or k.startswith(pre + "embed_tokens") or k.startswith(pre + "embeddings.")
                   for k in keys):
                self.prefix = pre
                break
        # names outside the decoder body (``language_model.lm_head`` next to
        # ``language_model.model.layers``)
        self.outer = self.prefix[:-len("model.")] if self.prefix.endswith("model.") else self.prefix
        self.used = set()

    def _key(self, name):
        for k in (self.prefix + name, name, self.outer + name):
            if k in self.t:
                return k
        return None

    def has(self, name):
        return self._key(name) is not None

    def raw(self, name):
        key = self._key(name) or name
        self.used.add(key)
        return self.t[key]

    def _qparams(self, base):
        q = self.q
        per = q.get(base) if isinstance(q.get(base), dict) else None
        src = per or q
        return src.get("group_size", 64), src.get("bits", 4), src.get("mode", "affine")

    def linear(self, base, required=True, packed=True):
        """Weight of a linear layer `base` (without the .weight suffix). Affine
        2-8-bit weights stay packed (QuantizedWeight) when the view keeps
        quantised weights and `packed`; everything else is dequantised. A
        Prism Hadamard module (``.signs``) comes back as a RotatedWeight whose
        rotation is its Hadamard transform."""
        w = self._linear(base, required, packed)
        if w is not None and self.hadamard is not None and self.has(base + ".signs"):
            from ..ops.rotation import RotatedWeight

            if isinstance(w, QuantizedWeight) and w.shape[0] % 8:  # the packed kernels tile 8 output rows
                w = w.dequantize(torch.float32).to(self.dtype)
            return RotatedWeight([(self.hadamard.transform(w.shape[1]), w)])
        return w

    def embedding(self, base):
        """Dense embedding table; a Prism Hadamard embedding is inverse-
        transformed once here, so lookups need no transform."""
        w = self._linear(base, True, False)
        if self.hadamard is not None and self.has(base + ".signs"):
            from .prism import inverse_embedding

            w = inverse_embedding(w.float(), self.hadamard.transform(w.shape[1])).to(self.dtype)
        return w

    def _linear(self, base, required=True, packed=True):
        wname = base + ".weight"
        if self.has(base + ".qweight"):  # AutoAWQ packing (ParoQuant checkpoints)
            return self._awq(base, packed)
        if not self.has(wname):
            if self.has(base):  # bare parameter (e.g. gpt-oss experts.gate_up_proj)
                return self.raw(base).to(self.dtype)
            if required:
                raise KeyError(f"missing weight {self.prefix + wname}")
            return None
        w = self.raw(wname)
        if self.has(base + ".weight_scale"):  # NVIDIA ModelOpt NVFP4 / FP8
            return self._modelopt(base, w, packed)
        if self.has(base + ".scales"):
            gs, bits, mode = self._qparams(base)  # MLX quantisation
            s = self.raw(base + ".scales")
            b = self.raw(base + ".biases") if self.has(base + ".biases") else None
            if self.keep_quantized and packed:
                qw = _packed(w, s, b, mode, bits, gs)
                if qw is not None:
                    return qw
            return quant.dequantize(w, s, b, mode, gs, bits, torch.float32).to(self.dtype)
        return w.to(self.dtype)

    def _awq(self, base, packed):
        """AutoAWQ 4-bit weight -> affine QuantizedWeight; with ParoQuant
        rotation tensors (``theta``, ``pairs``, ``channel_scales``) a
        :class:`RotatedWeight` that rotates the activations first."""
        from ..ops.rotation import PairwiseRotation, RotatedWeight, awq_to_quantized

        gs = self.q.get("group_size", 128)
        qw = awq_to_quantized(self.raw(base + ".qweight"), self.raw(base + ".qzeros"), self.raw(base + ".scales"), gs)
        w = qw if (self.keep_quantized and packed) else qw.dequantize(torch.float32).to(self.dtype)
        if self.has(base + ".theta"):
            cs = self.raw(base + ".channel_scales") if self.has(base + ".channel_scales") else None
            rot = PairwiseRotation(self.raw(base + ".theta"), self.raw(base + ".pairs"), cs)
            return RotatedWeight([(rot, w)])
        return w

    def _rotation(self, prefix):
        """A shared rotation (MoE experts: ``experts.{gate_up,down}_weight_*``)."""
        from ..ops.rotation import PairwiseRotation

        if not self.has(prefix + "theta"):
            return None
        cs = self.raw(prefix + "channel_scales") if self.has(prefix + "channel_scales") else None
        return PairwiseRotation(self.raw(prefix + "theta"), self.raw(prefix + "pairs"), cs)

    def _modelopt(self, base, w, packed):
        """ModelOpt checkpoints: NVFP4 (uint8 pairs of e2m1 codes, e4m3 block
        scales per 16 inputs, fp32 ``weight_scale_2``) stays packed for the
        e2m1 kernels when the view keeps quantised weights; FP8 (e4m3 weights
        with a per-tensor or per-output-channel ``weight_scale``) is
        dequantised. ``input_scale`` (activation quantisation) is not used:
        activations stay bf16."""
        ws = self.raw(base + ".weight_scale")
        if w.dtype == torch.uint8 and self.has(base + ".weight_scale_2"):
            g2 = float(self.raw(base + ".weight_scale_2").float().reshape(-1)[0])
            b = w.to(torch.int32)
            codes = torch.stack([b & 0x0F, b >> 4], -1).reshape(w.shape[0], -1)
            qw = QuantizedWeight.from_nvfp4(codes, ws, g2)
            if self.keep_quantized and packed and qw.shape[1] % 64 == 0 and qw.shape[0] % 8 == 0:
                return qw
            return qw.dequantize(torch.float32).to(self.dtype)
        s = ws.float()
        if s.numel() > 1:
            s = s.reshape(-1, 1)
        return (w.float() * s).to(self.dtype)

    def vec(self, name, required=False):
        if not self.has(name):
            if required:
                raise KeyError(name)
            return None
        return self.raw(name).to(self.dtype)


def _rows(w, idx: torch.Tensor):
    if _rotated([w]):
        from ..ops.rotation import RotatedWeight

        assert len(w.parts) == 1, "row selection of a single rotated projection"
        r, inner = w.parts[0]
        return RotatedWeight([(r, _rows(inner, idx))])
    return w.select_rows(idx) if isinstance(w, QuantizedWeight) else w.index_select(0, idx)


def _load_mla(ck: CheckpointView, cfg, L, a, norm):
    """Multi-head latent attention projections (DeepSeek V2 / V3, GLM-4.7-Flash).
    MLX conversions that split kv_b_proj into per-head ``embed_q`` [H, kv_lora,
    qk_nope] and ``unembed_out`` [H, v_head, kv_lora]
    (MLXLLM/Models/GLM4MOELite.swift:523-570) are put back together as
    kv_b [H * (qk_nope + v_head), kv_lora]."""
    from ..models import mla

    ql, kl, nope, rope_d, vd = mla.mla_dims(cfg)
    H = cfg.num_heads
    if ck.has(a + "q_a_proj.weight"):
        L.mla_q_a = ck.linear(a + "q_a_proj", packed=False)
        L.mla_q_a_norm = norm(a + "q_a_layernorm.weight")
        L.mla_q_b = ck.linear(a + "q_b_proj", packed=False)
    else:
        L.mla_q_b = ck.linear(a + "q_proj", packed=False)
    L.mla_kv_a = ck.linear(a + "kv_a_proj_with_mqa", packed=False)
    L.mla_kv_a_norm = norm(a + "kv_a_layernorm.weight")
    if ck.has(a + "kv_b_proj.weight"):
        L.mla_kv_b = ck.linear(a + "kv_b_proj", packed=False)
    else:
        wk = ck.linear(a + "embed_q", packed=False).reshape(H, kl, nope)
        wv = ck.linear(a + "unembed_out", packed=False).reshape(H, vd, kl)
        L.mla_kv_b = torch.cat([wk.transpose(1, 2), wv], 1).reshape(H * (nope + vd), kl).contiguous()
    L.wo = ck.linear(a + "o_proj", packed=False)


def _load_attention(ck: CheckpointView, cfg, L, a, norm, r, w):
    """q|k|v (and, for gated attention, the output gate after v), biases,
    q/k norms, o_proj and sinks of one attention layer."""
    if cfg.extra.get("mla"):
        if w > 1:
            raise NotImplementedError("multi-head latent attention loads without tensor parallelism")
        return _load_mla(ck, cfg, L, a, norm)
    if cfg.attn_output_gate:
        # q_proj rows per head: [q (D) | gate (D)] -> q | k | v | gate
        assert w == 1, "gated attention loads without tensor parallelism"
        qg = ck.linear(a + "q_proj")
        D, H = cfg.head_dim, cfg.num_heads
        qi = torch.tensor([h * 2 * D + d for h in range(H) for d in range(D)])
        L.wqkv = _cat_rows([_rows(qg, qi), ck.linear(a + "k_proj"), ck.linear(a + "v_proj"), _rows(qg, qi + D)])
    else:
        if cfg.extra.get("fused_qkv"):
            qkv = ck.linear(a + "qkv_proj", packed=False)
            qw, kw, vw = torch.split(qkv, [cfg.q_size, cfg.kv_size, cfg.kv_size], 0)
        else:
            qw, kw, vw = ck.linear(a + "q_proj"), ck.linear(a + "k_proj"), ck.linear(a + "v_proj")
        L.wqkv = _cat_rows([_shard_rows(qw, r, w), _kv_rows(kw, cfg, r, w), _kv_rows(vw, cfg, r, w)])
    if cfg.attention_bias:
        qb, kb, vb = ck.vec(a + "q_proj.bias"), ck.vec(a + "k_proj.bias"), ck.vec(a + "v_proj.bias")
        if qb is not None:
            L.bqkv = torch.cat([_shard_rows(qb, r, w), _kv_rows(kb, cfg, r, w), _kv_rows(vb, cfg, r, w)], 0)
    if cfg.qk_norm or cfg.qk_norm_full:
        if cfg.qk_norm_full and w > 1:
            raise NotImplementedError("q/k norms over the whole projection need every head on one rank")
        L.q_norm = norm(a + "q_norm.weight")
        L.k_norm = norm(a + "k_norm.weight")
    L.wo = _shard_cols(ck.linear(a + "o_proj"), r, w)
    if cfg.o_bias:
        L.bo = ck.vec(a + "o_proj.bias")
    if cfg.attention_sinks:
        s = ck.vec(a + "sinks")
        L.sinks = _shard_rows(s.float(), r, w) if s is not None else torch.zeros(cfg.num_heads // w)


def _load_linear_attn(ck: CheckpointView, cfg, L, p):
    """Gated DeltaNet weights as the fused in-projection q | k | v | z | b | a.
    Qwen3-Next packs in_proj_qkvz / in_proj_ba per key head ([q, k, v..., z...]
    and [b..., a...] per head, MLXLLM/Models/Qwen3Next.swift:225-260); Qwen 3.5
    has separate in_proj_qkv / z / b / a (Qwen35.swift:255)."""
    la = p + "linear_attn."
    Hk, Dk, Hv, Dv = cfg.gdn_dims
    vpk = Hv // Hk
    if ck.has(la + "in_proj_qkvz.weight"):
        W = ck.linear(la + "in_proj_qkvz")
        blk = 2 * Dk + 2 * vpk * Dv

        def sec(off, n):
            return torch.tensor([h * blk + off + j for h in range(Hk) for j in range(n)])

        BA = ck.linear(la + "in_proj_ba")
        bi = torch.tensor([h * 2 * vpk + j for h in range(Hk) for j in range(vpk)])
        parts = [_rows(W, sec(0, Dk)), _rows(W, sec(Dk, Dk)), _rows(W, sec(2 * Dk, vpk * Dv)),
                 _rows(W, sec(2 * Dk + vpk * Dv, vpk * Dv)), _rows(BA, bi), _rows(BA, bi + vpk)]
    else:
        parts = [ck.linear(la + "in_proj_qkv"), ck.linear(la + "in_proj_z"), ck.linear(la + "in_proj_b"),
                 ck.linear(la + "in_proj_a")]
    if len({type(t) for t in parts}) > 1 or any(isinstance(t, QuantizedWeight) and t.shape[0] % 8 for t in parts):
        parts = [t.dequantize(torch.float32) if isinstance(t, QuantizedWeight) else t for t in parts]
    L.wqkv = _cat_rows(parts)
    cw = ck.raw(la + "conv1d.weight").float()
    L.conv_w = (cw[:, 0, :] if cw.shape[-1] != 1 else cw[:, :, 0]).contiguous()
    L.A_log = ck.raw(la + "A_log").float()
    L.dt_bias = ck.raw(la + "dt_bias").float()
    L.gdn_norm = ck.vec(la + "norm.weight", required=True).float()
    L.wo = ck.linear(la + "out_proj")


_LFM2_RENAMES = ((".feed_forward.expert_bias", ".mlp.gate.e_score_correction_bias"),
                 (".feed_forward.gate.", ".mlp.gate."), (".feed_forward.experts.", ".mlp.experts."),
                 (".self_attn.out_proj.", ".self_attn.o_proj."), (".self_attn.q_layernorm.", ".self_attn.q_norm."),
                 (".self_attn.k_layernorm.", ".self_attn.k_norm."), (".operator_norm.", ".input_layernorm."),
                 (".ffn_norm.", ".post_attention_layernorm."), (".feed_forward.w1.", ".mlp.gate_proj."),
                 (".feed_forward.w3.", ".mlp.up_proj."), (".feed_forward.w2.", ".mlp.down_proj."),
                 ("embedding_norm.", "norm."))


def _lfm2_names(tensors: dict) -> dict:
    """LFM2 tensor names -> the decoder's (operator / ffn norms, w1/w3/w2,
    out_proj and q/k layernorms of the attention layers, embedding_norm as
    the final norm; LFM2-MoE routers, expert biases and experts); the
    short-conv layers keep ``conv.*``."""
    out = {}
    for k, v in tensors.items():
        for a, b in _LFM2_RENAMES:
            k = k.replace(a, b)
        if ".mlp.experts." in k:
            k = k.replace(".w1.", ".gate_proj.").replace(".w3.", ".up_proj.").replace(".w2.", ".down_proj.")
        out[k] = v
    return out


_BAILING_RENAMES = (("word_embeddings.", "embed_tokens."), (".attention.query_key_value.", ".self_attn.qkv_proj."),
                    (".attention.dense.", ".self_attn.o_proj."), (".attention.query_layernorm.", ".self_attn.q_norm."),
                    (".attention.key_layernorm.", ".self_attn.k_norm."), (".mlp.gate.gate_proj.", ".mlp.gate."),
                    (".mlp.gate.expert_bias", ".mlp.gate.e_score_correction_bias"))


def _renamed(tensors: dict, renames) -> dict:
    out = {}
    for k, v in tensors.items():
        for a, b in renames:
            k = k.replace(a, b)
        out[k] = v
    return out


def _load_mamba(ck: CheckpointView, cfg, L, mx):
    """Mamba-2 mixer weights. The in-projection's z | x | B | C | dt rows
    (MLXLLM/Models/NemotronH.swift:140-150) are reordered to C | B | x | z |
    dt, the layout of the recurrent kernels (C and B take the q and k
    places), and the conv channels x | B | C to C | B | x."""
    G, N, H, P = cfg.gdn_dims
    I, GN = H * P, G * N
    ar = torch.arange
    idx = torch.cat([ar(2 * I + GN, 2 * I + 2 * GN), ar(2 * I, 2 * I + GN), ar(I, 2 * I), ar(0, I),
                     ar(2 * I + 2 * GN, 2 * I + 2 * GN + H)])
    L.wqkv = _rows(ck.linear(mx + "in_proj"), idx)
    if ck.has(mx + "in_proj.bias"):
        L.bqkv = ck.vec(mx + "in_proj.bias")[idx]
    cidx = torch.cat([ar(I + GN, I + 2 * GN), ar(I, I + GN), ar(0, I)])
    cw = ck.raw(mx + "conv1d.weight").float()
    L.conv_w = (cw[:, 0, :] if cw.shape[-1] != 1 else cw[:, :, 0])[cidx].contiguous()
    if ck.has(mx + "conv1d.bias"):
        L.conv_b = ck.raw(mx + "conv1d.bias").float()[cidx].contiguous()
    L.A_log = ck.raw(mx + "A_log").float()
    L.dt_bias = ck.raw(mx + "dt_bias").float()
    L.ssm_D = ck.raw(mx + "D").float()
    L.gdn_norm = ck.vec(mx + "norm.weight", required=True)
    L.wo = ck.linear(mx + "out_proj")
    if ck.has(mx + "out_proj.bias"):
        L.bo = ck.vec(mx + "out_proj.bias")


def _packed(w, s, b, mode, bits, gs):
    """A packed QuantizedWeight for MLX affine 4/8-bit or MXFP4 weights the
    kernels serve (stacked experts [E, N, ...] keep num_experts), else None."""
    E = w.shape[0] if w.dim() == 3 else 0
    w2 = w.reshape(-1, w.shape[-1])
    s2 = s.reshape(-1, s.shape[-1])
    if mode == "affine" and b is not None and bits in CARRIED_BITS and gs in SUPPORTED_GROUPS:
        qw = QuantizedWeight.from_mlx(w2, s2.to(torch.bfloat16), b.reshape(-1, b.shape[-1]).to(torch.bfloat16), bits,
                                      gs)
    elif mode == "mxfp4" and bits == 4 and gs == 32:
        qw = QuantizedWeight.from_mlx_mxfp4(w2, s2)
    else:
        return None
    qw.num_experts = E
    return qw


def _stack(parts):
    if isinstance(parts[0], QuantizedWeight):
        return QuantizedWeight.stack_experts(parts)
    return torch.stack(parts)


def _expert(w, e):
    return w.expert(e) if isinstance(w, QuantizedWeight) else w[e]


def _shard_rows(w, rank, world):
    if w is None or world == 1:
        return w
    n = w.shape[0] // world
    if isinstance(w, QuantizedWeight):
        return w.rows(rank * n, (rank + 1) * n)
    return w[rank * n:(rank + 1) * n]


def _shard_cols(w, rank, world):
    if w is None or world == 1:
        return w
    n = w.shape[-1] // world
    if isinstance(w, QuantizedWeight):
        return w.cols(rank * n, (rank + 1) * n)
    return w[..., rank * n:(rank + 1) * n]


def _kv_rows(w, cfg, rank, world):
    """K or V projection rows for this rank (heads split, or replicated when KVH < world)."""
    if w is None or world == 1:
        return w
    D = cfg.head_dim
    if cfg.num_kv_heads >= world:
        return _shard_rows(w, rank, world)
    h = (rank * cfg.num_kv_heads) // world
    if isinstance(w, QuantizedWeight):
        return w.rows(h * D, (h + 1) * D)
    return w[h * D:(h + 1) * D]


def load_model(path: str, device="cuda", dtype=torch.bfloat16, tp: TensorParallel | None = None,
               config_overrides: dict | None = None, keep_quantized: bool = True, with_mtp: bool = False):
    """Load a model directory (config.json + *.safetensors). Returns (model, hf_config).
    MLX affine 4/8-bit projections stay packed unless `keep_quantized` is False.
    `with_mtp`: also load the checkpoint's MTP head (Qwen 3.5 ``mtp.*``,
    DeepSeek V3 / GLM nextn layers, MiMo ``mtp_layers``) as ``model.mtp_head``
    (None when the checkpoint has none)."""
    with open(os.path.join(path, "config.json")) as f:
        hf = json.load(f)
    hadamard = None
    if prism.is_prism(hf):
        info = prism.parse_config(hf)
        hadamard = prism.HadamardMetadata.read(path)
        hf = prism.text_config(hf)
    cfg = build_config(hf)
    for k, v in (config_overrides or {}).items():
        setattr(cfg, k, v)
    tensors, _ = load_safetensors(path)
    if hadamard is not None:
        prism.validate(info, hadamard, tensors)
    model = build_from_tensors(cfg, tensors, device, dtype, tp, keep_quantized=keep_quantized, hadamard=hadamard)
    if hf.get("vision_config") and hf.get("model_type") in ("qwen2_vl", "qwen2_5_vl", "qwen3_vl"):
        model = _attach_vision(model, cfg, hf, tensors, device, dtype)
    elif hf.get("vision_config") and hf.get("model_type") in ("gemma3", "paligemma", "idefics3", "smolvlm"):
        model = _attach_siglip(model, cfg, hf, tensors, device, dtype, path)
    if with_mtp:
        from ..models.mtp import load_mtp

        model.mtp_head = load_mtp(model, tensors)
    return model, hf


def _attach_vision(lm, cfg, hf, tensors, device, dtype):
    """Qwen2-VL / Qwen2.5-VL: the loaded language model plus its vision tower
    (``visual.*`` / ``model.visual.*``) as one :class:`Qwen2VLModel`."""
    from ..models.vision import QwenVisionTower, VisionConfig
    from ..models.vlm import Qwen2VLModel

    tc = hf.get("text_config") or {}
    rs = hf.get("rope_scaling") or tc.get("rope_scaling") or tc.get("rope_parameters") or {}
    mt = hf.get("model_type")
    kind = {"qwen2_5_vl": "qwen2_5", "qwen3_vl": "qwen3"}.get(mt, "qwen2")
    vcfg = VisionConfig.from_hf(hf["vision_config"], cfg.hidden_size, kind)
    if kind == "qwen3":
        from ..models.vlm import Qwen3VLModel

        m = Qwen3VLModel(cfg, vcfg, device, dtype, hf.get("image_token_id", 151655), hf.get("video_token_id", 151656),
                         rs.get("mrope_section", (24, 20, 20)))
    else:
        m = Qwen2VLModel(cfg, vcfg, device, dtype, hf.get("image_token_id", 151655),
                         hf.get("video_token_id", 151656), rs.get("mrope_section", (16, 24, 24)))
    m.embed, m.norm, m.lm_head, m.layers = lm.embed, lm.norm, lm.lm_head, lm.layers
    m.vision = QwenVisionTower.from_tensors(vcfg, tensors, device, dtype)
    return m


def _attach_siglip(lm, cfg, hf, tensors, device, dtype, path=None):
    """SigLIP-tower VLMs: the loaded language model plus the vision tower and
    the connector as one :class:`..models.siglip.SiglipVLM` - Gemma 3 (pooled
    projector ``multi_modal_projector.*``), PaliGemma (``multi_modal_projector
    .linear``), Idefics3 / SmolVLM (``connector.modality_projection.proj``)."""
    from ..models.siglip import SiglipConfig, SiglipVisionTower, SiglipVLM

    mt = hf["model_type"]
    vc = hf["vision_config"]
    vcfg = SiglipConfig.from_hf(vc)
    itok = hf.get("image_token_index", hf.get("image_token_id"))
    if mt == "gemma3":
        m = SiglipVLM(cfg, vcfg, device, dtype, "gemma3", itok if itok is not None else 262144,
                      hf.get("mm_tokens_per_image", 256))
    elif mt == "paligemma":
        m = SiglipVLM(cfg, vcfg, device, dtype, "paligemma", itok if itok is not None else 257152,
                      vc.get("num_image_tokens", vcfg.grid * vcfg.grid))
    else:
        sf = int(hf.get("scale_factor", 2))
        m = SiglipVLM(cfg, vcfg, device, dtype, "idefics3", itok if itok is not None else 128257,
                      (vcfg.grid // sf) ** 2, sf)
    m.embed, m.norm, m.lm_head, m.layers = lm.embed, lm.norm, lm.lm_head, lm.layers
    m.vision = SiglipVisionTower.from_tensors(vcfg, tensors, device, dtype)

    def find(*names):
        for n in names:
            for pre in ("model.multi_modal_projector.", "multi_modal_projector.", "model.connector.", "connector."):
                if pre + n in tensors:
                    return tensors[pre + n].to(device, dtype)
        return None

    if mt == "gemma3":
        m.proj_w = find("mm_input_projection_weight")
        m.proj_norm = find("mm_soft_emb_norm.weight")
    elif mt == "paligemma":
        m.proj_w, m.proj_b = find("linear.weight"), find("linear.bias")
    else:
        m.proj_w = find("modality_projection.proj.weight")
    if m.proj_w is None:
        raise KeyError(f"no {mt} projector weights")
    if path is not None:  # processor: normalisation and (SmolVLM) tiling
        pp = os.path.join(path, "preprocessor_config.json")
        if os.path.exists(pp):
            with open(pp) as f:
                pc = json.load(f)
            m.image_mean = tuple(pc.get("image_mean", m.image_mean))
            m.image_std = tuple(pc.get("image_std", m.image_std))
            if mt == "smolvlm" and pc.get("do_image_splitting", True):
                m.tile_longest_edge = int((pc.get("size") or {}).get("longest_edge", 0))
    return m


def build_from_tensors(cfg: DecoderConfig, tensors: dict, device="cpu", dtype=torch.float32, tp=None,
                       keep_quantized: bool = False, hadamard=None):
    """Build a DecoderLM from checkpoint tensors. With `keep_quantized`, MLX
    affine 4/8-bit projections of dense layers stay packed and run through
    the dequantising GEMM; embeddings, MoE experts and other formats are
    dequantised."""
    tp = tp or TensorParallel()
    r, w = tp.rank, tp.world
    if cfg.linear_kind == "short_conv":
        tensors = _lfm2_names(tensors)
    if cfg.model_type == "bailing_moe":
        tensors = _renamed(tensors, _BAILING_RENAMES)
    if cfg.model_type == "phi":
        return _build_phi(cfg, tensors, device, dtype)
    q = cfg.quantization if isinstance(cfg.quantization, dict) else None
    ck = CheckpointView(tensors, q, torch.float32, keep_quantized=keep_quantized and bool(q), hadamard=hadamard)
    if cfg.extra.get("gemma4"):
        from ..models import gemma4

        if tp.world != 1:
            raise NotImplementedError("Gemma 4 loads without tensor parallelism")
        return gemma4.build_from_tensors(cfg, ck, tensors, device, dtype)
    if cfg.layer_types and any(cfg.is_linear(i) for i in range(cfg.num_layers)):
        assert tp.world == 1, "hybrid (linear-attention) models load without tensor parallelism"
        # HF-format Qwen3-Next / 3.5 checkpoints store zero-centred layer norms
        # and conv taps as [C, 1, K]; MLX-converted ones already hold 1 + w
        # and [C, K, 1] (the rule of MLXLLM/Models/Qwen3Next.swift:807-855)
        li = next(i for i in range(cfg.num_layers) if cfg.is_linear(i))
        if cfg.linear_kind == "gdn" and ck.raw(f"layers.{li}.linear_attn.conv1d.weight").shape[-1] != 1:
            cfg.norm_offset_one = True
    m = DecoderLM(cfg, "cpu", torch.float32, tp=tp)
    off = 1.0 if cfg.norm_offset_one else 0.0

    def norm(name):
        v = ck.vec(name, required=True).float()
        return v + off

    m.embed = ck.embedding("embed_tokens" if ck.has("embed_tokens.weight") else "embeddings")
    m.norm = norm("norm.weight" if ck.has("norm.weight") else "norm_f.weight")
    if cfg.norm_kind == "layernorm":
        m.norm_b = ck.vec("norm.bias")
    if hadamard is not None and not ck.has("lm_head.weight") and ck.has("embed_tokens.signs"):
        m.lm_head = ck.linear("embed_tokens")  # tied head: packed table behind the forward transform
    elif ck.has("diffusion_head.weight"):  # Nemotron-Labs-Diffusion
        m.lm_head = ck.linear("diffusion_head")
    elif cfg.tie_word_embeddings or not (ck.has("lm_head.weight") or "lm_head.weight" in tensors):
        m.lm_head = m.embed
    else:
        m.lm_head = ck.linear("lm_head") if ck.has("lm_head.weight") else ck.linear("lm_head", False)
        if isinstance(m.lm_head, QuantizedWeight) and (m.lm_head.shape[0] % 8):
            m.lm_head = m.lm_head.dequantize(torch.float32)
        if m.lm_head is None:
            key = "lm_head.weight"
            m.lm_head = tensors[key].float()
    hd = cfg.head_dim
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        L = LayerWeights()
        if cfg.layer_blocks:  # one block per layer (NemotronH / Mamba2): norm + mixer
            L.block = cfg.block(i)
            L.ln1 = norm(p + "norm.weight")
            L.linear = cfg.is_linear(i)
            mx = p + "mixer."
            if L.block == "ffn":  # non-gated relu^2 MLP
                L.moe = False
                L.wgu = _shard_rows(ck.linear(mx + "up_proj"), r, w)
                L.wd = _shard_cols(ck.linear(mx + "down_proj"), r, w)
                if cfg.mlp_bias:
                    L.bgu, L.bd = ck.vec(mx + "up_proj.bias"), ck.vec(mx + "down_proj.bias")
            elif L.linear:
                _load_mamba(ck, cfg, L, mx)
            else:
                _load_attention(ck, cfg, L, mx, norm, r, w)
            m.layers.append(L)
            continue
        n_in, n_post = cfg.extra.get("norm_names", ("input_layernorm", "post_attention_layernorm"))
        L.ln1 = norm(p + n_in + ".weight")
        if cfg.norm_kind == "layernorm":
            L.ln1_b = ck.vec(p + "input_layernorm.bias")
            L.ln2_b = ck.vec(p + "post_attention_layernorm.bias")
        if cfg.parallel_block:  # one norm feeds attention and MLP
            pass
        elif not cfg.pre_norms:  # post-sublayer norms only (OLMo 2/3, EXAONE 4)
            L.ln1 = None
            L.post_attn_norm = norm(p + "post_attention_layernorm.weight")
            L.post_ffn_norm = norm(p + "post_feedforward_layernorm.weight")
        elif cfg.post_norms:
            L.post_attn_norm = norm(p + "post_attention_layernorm.weight")
            L.ln2 = norm(p + "pre_feedforward_layernorm.weight")
            L.post_ffn_norm = norm(p + "post_feedforward_layernorm.weight")
        else:
            L.ln2 = norm(p + n_post + ".weight")
        L.linear = cfg.is_linear(i)
        if L.linear and cfg.linear_kind == "short_conv":  # LFM2: layers.{i}.conv.*
            mx = p + "conv."
            L.wqkv = ck.linear(mx + "in_proj")
            cw = ck.raw(mx + "conv.weight").float()
            L.conv_w = (cw[:, 0, :] if cw.shape[-1] != 1 else cw[:, :, 0]).contiguous()
            if ck.has(mx + "conv.bias"):
                L.conv_b = ck.raw(mx + "conv.bias").float()
            L.wo = ck.linear(mx + "out_proj")
            if ck.has(mx + "in_proj.bias"):
                L.bqkv = ck.vec(mx + "in_proj.bias")
            if ck.has(mx + "out_proj.bias"):
                L.bo = ck.vec(mx + "out_proj.bias")
        elif L.linear and cfg.linear_kind == "mamba2":  # Granite 4 hybrids: layers.{i}.mamba.*
            _load_mamba(ck, cfg, L, p + "mamba.")
        elif L.linear:
            _load_linear_attn(ck, cfg, L, p)
        else:
            _load_attention(ck, cfg, L, p + "self_attn.", norm, r, w)
        if cfg.is_moe(i):
            _load_moe(ck, cfg, L, p, r, w)
        else:
            mp = p + "mlp."
            if ck.has(p + "shared_mlp.input_linear.weight"):  # Granite 4 dense: [gate | up] rows
                mp = p + "shared_mlp."
                g, u = ck.linear(mp + "input_linear", packed=False).chunk(2, 0)
                L.moe = False
                L.wgu = interleave_gate_up(_shard_rows(g, r, w), _shard_rows(u, r, w))
                L.wd = _shard_cols(ck.linear(mp + "output_linear"), r, w)
                m.layers.append(L)
                continue
            if ck.has(mp + "c_fc.weight"):  # StarCoder2: non-gated GELU MLP with biases
                L.moe = False
                L.wgu, L.wd = ck.linear(mp + "c_fc"), ck.linear(mp + "c_proj")
                L.bgu, L.bd = ck.vec(mp + "c_fc.bias"), ck.vec(mp + "c_proj.bias")
                m.layers.append(L)
                continue
            if cfg.glu_epi == "xielu":  # Apertus: non-gated up -> xIELU -> down
                L.moe = False
                L.wgu = _shard_rows(ck.linear(mp + "up_proj"), r, w)
                L.wd = _shard_cols(ck.linear(mp + "down_proj"), r, w)
                L.act_params = torch.stack([ck.raw(mp + "act_fn." + n).float().reshape(())
                                            for n in ("alpha_p", "alpha_n", "beta", "eps")])
                m.layers.append(L)
                continue
            if cfg.extra.get("fused_gate_up"):
                gu = ck.linear(mp + "gate_up_proj", packed=False)
                g, u = gu.chunk(2, 0)
            else:
                g, u = ck.linear(mp + "gate_proj"), ck.linear(mp + "up_proj")
            L.moe = False
            L.wgu = interleave_gate_up(_shard_rows(g, r, w), _shard_rows(u, r, w))
            L.wd = _shard_cols(ck.linear(mp + "down_proj"), r, w)
            if cfg.mlp_bias:
                gb, ub = ck.vec(mp + "gate_proj.bias"), ck.vec(mp + "up_proj.bias")
                if gb is not None:
                    L.bgu = _interleave_dense(_shard_rows(gb, r, w)[:, None], _shard_rows(ub, r, w)[:, None])[:, 0]
                L.bd = ck.vec(mp + "down_proj.bias")
        m.layers.append(L)
    if cfg.norm_offset_one:
        cfg.norm_offset_one = False  # folded into the stored weights
        cfg.extra["norms_zero_centred"] = True  # the checkpoint stores w - 1 (MTP heads beside it too)
    _fold_multipliers(m, cfg)
    return m.clone_to(device, dtype)


def _scale(w, f: float):
    if w is None or f == 1.0:
        return w
    if isinstance(w, QuantizedWeight):
        try:
            return w.scaled(f)
        except ValueError:
            return w.dequantize(torch.float32) * f
    return w * f


def _fold_multipliers(m, cfg):
    """Granite-family multipliers folded into the weights: the residual
    branch scale into the output projections of every block (o_proj /
    out_proj, down / expert / shared outputs and their biases), and the
    logits divisor into the head (untied from the embedding when shared).
    Parity: MLXLLM/Models/Granite.swift and GraniteMoeHybrid.swift:430-442
    (residual + branch * residual_multiplier, logits / logits_scaling)."""
    rm = float(cfg.extra.get("residual_multiplier", 1.0))
    ls = float(cfg.extra.get("logits_scaling", 1.0))
    if rm != 1.0:
        for L in m.layers:
            for n in ("wo", "bo", "wd", "bd", "experts_d", "experts_d_b", "shared_d"):
                setattr(L, n, _scale(getattr(L, n), rm))
    if ls != 1.0:
        m.lm_head = _scale(m.lm_head, 1.0 / ls)  # a new tensor: the embedding keeps its values


def _load_moe(ck: CheckpointView, cfg, L, p, r, w):
    L.moe = True
    E = cfg.num_experts
    if cfg.model_type == "gpt_oss":
        mp = p + "mlp."
        L.router = ck.linear(mp + "router", packed=False)
        L.router_b = ck.vec(mp + "router.bias")
        packed = ck.keep_quantized and ck.has(mp + "experts.gate_up_proj_blocks")
        if packed:
            # HF MXFP4 blocks stay packed: rows are outputs, gate at even and
            # up at odd rows of gate_up
            gq = _mxfp4_packed(ck.raw(mp + "experts.gate_up_proj_blocks"), ck.raw(mp + "experts.gate_up_proj_scales"))
            dq = _mxfp4_packed(ck.raw(mp + "experts.down_proj_blocks"), ck.raw(mp + "experts.down_proj_scales"))
            F2 = gq.shape[0] // E
            even = torch.arange(0, F2, 2)
            L.experts_gu = QuantizedWeight.stack_experts([
                interleave_gate_up(_shard_rows(gq.expert(e).select_rows(even), r, w),
                                   _shard_rows(gq.expert(e).select_rows(even + 1), r, w)) for e in range(E)])
            L.experts_d = QuantizedWeight.stack_experts([_shard_cols(dq.expert(e), r, w) for e in range(E)])
        elif ck.has(mp + "experts.gate_up_proj_blocks"):
            blocks = ck.raw(mp + "experts.gate_up_proj_blocks")  # [E, 2F, K/32, 16] uint8
            scales = ck.raw(mp + "experts.gate_up_proj_scales")  # [E, 2F, K/32] uint8
            gu = _mxfp4_blocks(blocks, scales)  # [E, 2F, K]
            gu = gu.transpose(1, 2)  # -> [E, K, 2F] as the bf16 layout
            db = ck.raw(mp + "experts.down_proj_blocks")
            ds = ck.raw(mp + "experts.down_proj_scales")
            down = _mxfp4_blocks(db, ds).transpose(1, 2)  # [E, F, K]... as bf16 layout [E, F, K]
        else:
            gu = ck.raw(mp + "experts.gate_up_proj").float()  # [E, K, 2F] (gate even, up odd columns)
            down = ck.raw(mp + "experts.down_proj").float()  # [E, F, K]
        if not packed:
            g, u = gu[..., 0::2].transpose(1, 2), gu[..., 1::2].transpose(1, 2)  # [E, F, K]
            L.experts_gu = torch.stack([interleave_gate_up(_shard_rows(g[e], r, w), _shard_rows(u[e], r, w))
                                        for e in range(E)])
            L.experts_d = torch.stack([_shard_cols(down[e].t(), r, w) for e in range(E)])  # [E, K, F]
        gub = ck.vec(mp + "experts.gate_up_proj_bias")
        if gub is not None:
            gb, ub = gub[..., 0::2], gub[..., 1::2]
            L.experts_gu_b = torch.stack([interleave_gate_up(_shard_rows(gb[e], r, w)[:, None],
                                                             _shard_rows(ub[e], r, w)[:, None])[:, 0]
                                          for e in range(E)])
        L.experts_d_b = ck.vec(mp + "experts.down_proj_bias")
        return
    mixtral = cfg.extra.get("mixtral_names")
    mp = p + ("block_sparse_moe." if mixtral else "mlp.")
    if ck.has(p + "block_sparse_moe.router.layer.weight"):  # Granite 4 hybrids (HF names)
        _load_granite_moe(ck, cfg, L, p, r, w)
        return
    L.router = ck.linear(mp + "gate", packed=False)
    names = ("w1", "w3", "w2") if mixtral else ("gate_proj", "up_proj", "down_proj")
    # quantised experts stay packed when every expert's format is one the
    # grouped kernels serve (else all are dequantised)
    if ck.has(mp + "switch_mlp.gate_proj.weight"):
        g = ck.linear(mp + "switch_mlp.gate_proj")
        u = ck.linear(mp + "switch_mlp.up_proj")
        d = ck.linear(mp + "switch_mlp.down_proj")
        g, u, d = ([_expert(t, e) for e in range(E)] for t in (g, u, d))
    else:
        g, u, d = ([ck.linear(f"{mp}experts.{e}.{n}") for e in range(E)] for n in names)
    if not all(isinstance(t, QuantizedWeight) for t in g + u + d):
        g, u, d = ([t.dequantize(torch.float32).to(ck.dtype) if isinstance(t, QuantizedWeight) else t for t in x]
                   for x in (g, u, d))
    L.experts_gu = _stack([interleave_gate_up(_shard_rows(g[e], r, w), _shard_rows(u[e], r, w)) for e in range(E)])
    L.experts_d = _stack([_shard_cols(d[e], r, w) for e in range(E)])
    # ParoQuant: rotations shared by all experts of the layer
    L.experts_rot_in = ck._rotation(mp + "experts.gate_up_weight_")
    L.experts_rot_mid = ck._rotation(mp + "experts.down_weight_")
    if ck.has(mp + "gate.e_score_correction_bias"):  # sigmoid_group routers
        L.router_corr = ck.raw(mp + "gate.e_score_correction_bias").float()
    if cfg.shared_expert_intermediate_size:
        sp = mp + ("shared_experts." if ck.has(mp + "shared_experts.gate_proj.weight") else "shared_expert.")
        L.shared_gu = interleave_gate_up(_shard_rows(ck.linear(sp + "gate_proj"), r, w),
                                         _shard_rows(ck.linear(sp + "up_proj"), r, w))
        L.shared_d = _shard_cols(ck.linear(sp + "down_proj"), r, w)
        if ck.has(mp + "shared_expert_gate.weight"):
            L.shared_gate = ck.linear(mp + "shared_expert_gate", packed=False)


def _build_phi(cfg, tensors, device, dtype):
    """Phi-1.5 / Phi-2 (MLXLLM/Models/Phi.swift): q/k/v/dense and fc1/fc2 with
    biases, input_layernorm weight + bias, final_layernorm, biased lm_head."""
    ck = CheckpointView(tensors, None, torch.float32)
    m = DecoderLM(cfg, "cpu", torch.float32)
    m.embed = ck.linear("embed_tokens", packed=False)
    m.norm, m.norm_b = ck.vec("final_layernorm.weight", True), ck.vec("final_layernorm.bias", True)
    m.lm_head = ck.linear("lm_head", packed=False)
    m.lm_head_b = ck.raw("lm_head.bias").float() if ck.has("lm_head.bias") else None
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        L = LayerWeights()
        L.ln1, L.ln1_b = ck.vec(p + "input_layernorm.weight", True), ck.vec(p + "input_layernorm.bias", True)
        a = p + "self_attn."
        L.wqkv = torch.cat([ck.linear(a + n, packed=False) for n in ("q_proj", "k_proj", "v_proj")], 0)
        L.bqkv = torch.cat([ck.vec(a + n + ".bias", True) for n in ("q_proj", "k_proj", "v_proj")], 0)
        L.wo, L.bo = ck.linear(a + "dense", packed=False), ck.vec(a + "dense.bias", True)
        L.moe = False
        L.wgu, L.bgu = ck.linear(p + "mlp.fc1", packed=False), ck.vec(p + "mlp.fc1.bias", True)
        L.wd, L.bd = ck.linear(p + "mlp.fc2", packed=False), ck.vec(p + "mlp.fc2.bias", True)
        m.layers.append(L)
    return m.clone_to(device, dtype)


def _load_granite_moe(ck: CheckpointView, cfg, L, p, r, w):
    """GraniteMoeHybrid experts: router ``block_sparse_moe.router.layer``,
    ``input_linear`` [E, 2F, H] with the gate rows first, ``output_linear``
    [E, H, F], and the shared MLP ``shared_mlp.input_linear`` [2Fs, H] /
    ``output_linear`` (MLXLLM/Models/GraniteMoeHybrid.swift:270-350)."""
    mp = p + "block_sparse_moe."
    L.router = ck.linear(mp + "router.layer", packed=False)
    gu = ck.raw(mp + "input_linear.weight").to(ck.dtype)
    dn = ck.raw(mp + "output_linear.weight").to(ck.dtype)
    E = gu.shape[0]
    F = gu.shape[1] // 2
    L.experts_gu = torch.stack([interleave_gate_up(_shard_rows(gu[e, :F], r, w), _shard_rows(gu[e, F:], r, w))
                                for e in range(E)])
    L.experts_d = torch.stack([_shard_cols(dn[e], r, w) for e in range(E)])
    sp = p + "shared_mlp."
    if ck.has(sp + "input_linear.weight"):
        g, u = ck.linear(sp + "input_linear", packed=False).chunk(2, 0)
        L.shared_gu = interleave_gate_up(_shard_rows(g, r, w), _shard_rows(u, r, w))
        L.shared_d = _shard_cols(ck.linear(sp + "output_linear"), r, w)


def _mxfp4_packed(blocks, scales) -> QuantizedWeight:
    """HF MXFP4 expert stack (blocks [E, N, G, 16] uint8, two e2m1 codes per
    byte low nibble first; scales [E, N, G] e8m0) -> packed [E*N, 32G]."""
    E, N, G, _ = blocks.shape
    b = blocks.reshape(E * N, G * 16).to(torch.int32)
    codes = torch.stack([b & 0x0F, b >> 4], -1).reshape(E * N, G * 32)
    qw = QuantizedWeight.from_mxfp4(codes, scales.reshape(E * N, G))
    qw.num_experts = E
    return qw


def _mxfp4_blocks(blocks, scales):
    """HF MXFP4 (blocks [..., G, 16] uint8 with two e2m1 codes per byte, scales [..., G] e8m0) -> float."""
    lo = (blocks & 0x0F).to(torch.int64)
    hi = (blocks >> 4).to(torch.int64)
    codes = torch.stack([lo, hi], -1).reshape(*blocks.shape[:-1], 32)
    v = quant.E2M1[codes] * quant.e8m0_to_float(scales.to(torch.int64))[..., None]
    return v.reshape(*blocks.shape[:-2], -1)


def load_tokenizer(path: str):
    """A local HF tokenizer (no network), or None when the directory has none."""
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(path, local_files_only=True, trust_remote_code=False)
    except Exception:
        return None


def eos_token_ids(path: str, hf: dict, tokenizer=None) -> set[int]:
    ids = set()
    for src in (hf, _read_json(os.path.join(path, "generation_config.json"))):
        e = (src or {}).get("eos_token_id")
        if isinstance(e, int):
            ids.add(e)
        elif isinstance(e, list):
            ids.update(int(x) for x in e)
    if tokenizer is not None and getattr(tokenizer, "eos_token_id", None) is not None:
        ids.add(int(tokenizer.eos_token_id))
    return ids


def _read_json(p):
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


_ = math
