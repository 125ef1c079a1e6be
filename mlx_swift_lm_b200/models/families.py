"""Model-family adapters: HF/MLX ``config.json`` -> :class:`DecoderConfig`, and
checkpoint tensor names -> the fused decoder's weights.

Registry parity with MLXLLM/LLMModelFactory.swift:71-143 (``model_type`` keys).
Each adapter states the few switches in which its family differs from the
Llama baseline; :func:`build_config` handles the shared keys.
"""
from __future__ import annotations

import math

from .config import DecoderConfig

FAMILIES: dict[str, dict] = {}


def register(*model_types, **traits):
    for mt in model_types:
        FAMILIES[mt] = dict(traits)


# --- the registry -----------------------------------------------------------------
register("llama", "mistral", "smollm3", "helium", "granite", "hunyuan_v1_dense",
         "ernie4_5", "internlm2", "minicpm", "nanbeige", "laguna", "acereason", "mellum")
# architectures whose distinguishing blocks are not built: refused instead of loaded wrongly
_REFUSED: dict[str, str] = {}
# Apertus: Llama body with per-head q/k norms and a non-gated xIELU MLP (learned per-layer scalars)
register("apertus", qk_norm=True, apertus=True)
# post-sublayer norms only (no input norms), q/k RMSNorm over the whole projection
register("olmo2", "olmo3", post_only_norms=True, qk_norm_full=True)
# post-sublayer norms only, per-head q/k norms, local (L) / global (G) layer pattern, NoPE global layers
register("exaone4", post_only_norms=True, qk_norm=True, exaone4=True)
register("qwen2")  # q/k/v biases
register("mimo")  # Xiaomi MiMo: the Qwen2 body (its MTP layers are not loaded)
register("qwen2_vl", vlm="qwen2_vl")  # the language model of Qwen2-VL (q/k/v biases, M-RoPE)
register("qwen2_5_vl", vlm="qwen2_vl")  # Qwen2.5-VL: the same language model; window-attention vision tower
# Qwen3-VL: the Qwen3 language model (interleaved M-RoPE, deepstack rows in models/vlm.py)
register("qwen3_vl", "qwen3_vl_text", qk_norm=True, vlm="qwen3_vl")
register("qwen3", qk_norm=True)
register("qwen3_moe", qk_norm=True, moe=True)
register("qwen3_next", qk_norm=True, moe=True, hybrid=True)
register("qwen3_5", "qwen3_5_text", "qwen3_8", "qwen3_8_text", qk_norm=True, hybrid=True)
register("qwen3_5_moe", "qwen3_8_moe", qk_norm=True, moe=True, hybrid=True)
register("mixtral", moe=True, mixtral_names=True)
register("phimoe", moe=True, mixtral_names=True)
register("olmoe", moe=True, qk_norm=True)
register("gemma", gemma=1)
register("gemma2", gemma=2)
register("gemma3", "gemma3_text", gemma=3)
register("gemma4", "gemma4_text", gemma4=True)  # per-kind head dims, shared KV, per-layer inputs, MoE block
register("phi3", fused_qkv=True, fused_gate_up=True)
register("gpt_oss", gpt_oss=True)
register("glm4", fused_gate_up=True)
register("glm4_moe", moe=True, deepseek_router=True)  # GLM-4.5 / 4.6 / 4.7
# multi-head latent attention + DeepSeek routing (DeepSeek V2 / V3, GLM-4.7-Flash)
register("deepseek_v2", "deepseek_v3", "glm4_moe_lite", moe=True, deepseek_router=True, mla=True)
register("mistral3", "ministral3")  # the text model of Mistral 3 / Ministral 3 (Llama-4 query scaling)
# Ministral 3 backbone under ``encoder.*`` with a ``diffusion_head``; block
# mask-diffusion decoding (engine/block_diffusion.py)
register("nemotron_labs_diffusion", diffusion=True)
# Mamba-2 hybrids: one block per layer (M mamba, * attention, - MLP), and pure Mamba-2
register("nemotron_h", ssm="nemotron_h")
# IBM Granite 4 hybrids: Mamba-2 or attention mixer + MoE (top-k softmax over the k) + shared MLP per layer
register("granitemoehybrid", ssm="granite", moe=True, mixtral_names=False)
register("mamba2", ssm="mamba2")
register("lfm2", lfm2=True, qk_norm=True)
# LFM2-MoE: LFM2 layers whose FFN is a sigmoid-routed MoE (expert-bias corrected selection)
# after `num_dense_layers` dense ones
register("lfm2_moe", lfm2=True, qk_norm=True, lfm2_moe=True)
# Ling (Bailing MoE): fused query_key_value, optional q/k norms, partial rotary, sigmoid group-limited
# routing with expert bias, shared experts after `first_k_dense_replace` dense layers
register("bailing_moe", fused_qkv=True, bailing=True)
register("phi", phi2=True)  # Phi-1.5 / Phi-2: parallel attention + MLP, LayerNorm, partial rotary  # Liquid LFM2: short-conv / attention hybrid

_NEMOTRON_BLOCKS = {"mamba": "M", "attention": "*", "mlp": "-", "moe": "E"}


def _ssm_dt_limits(hf: dict) -> tuple[float, float]:
    """Execution limits of dt: ``time_step_limit`` ([min] or [min, max]),
    else ``time_step_limit_min`` / ``_max``, else ``time_step_min`` /
    ``_max``, else (0, inf) - the resolution order of
    MLXLLM/Models/NemotronH.swift:2252-2280."""
    lim = hf.get("time_step_limit")
    if isinstance(lim, (list, tuple)) and lim:
        if len(lim) > 2:
            raise ValueError("time_step_limit requires one or two values")
        lo, hi = float(lim[0]), float(lim[-1])
    else:
        lo = hf.get("time_step_limit_min", hf.get("time_step_min", 0.0))
        hi = hf.get("time_step_limit_max", hf.get("time_step_max", float("inf")))
        lo, hi = float(lo), float(hi)
    if not (math.isfinite(lo) and lo >= 0 and hi >= lo):
        raise ValueError(f"invalid dt limits ({lo}, {hi})")
    return lo, hi


def _ssm_prepare(hf: dict, kind: str) -> dict:
    """Fill the attention keys a pure / hybrid SSM config may omit."""
    hf = dict(hf)
    if kind == "granite":
        return hf
    if kind == "mamba2":
        hf.setdefault("num_attention_heads", 1)
        hf.setdefault("num_key_value_heads", 1)
        hf["ssm_head_dim"] = hf["head_dim"]  # the SSM head dim; no attention layers
        hf["head_dim"] = 64
        hf.setdefault("intermediate_size", 0)
        hf["rms_norm_eps"] = hf.get("layer_norm_epsilon", 1e-5)
    else:
        hf["rms_norm_eps"] = hf.get("layer_norm_epsilon", hf.get("norm_eps", 1e-5))
    return hf


def _ssm_config(cfg: DecoderConfig, hf: dict, kind: str):
    """Mamba-2 mixer geometry and the per-layer block layout."""
    if kind == "mamba2":
        H, P = hf["num_heads"], hf["ssm_head_dim"]
        N = hf.get("ssm_state_size", hf.get("state_size", 128))
        pattern = "M" * cfg.num_layers
        norm_groups = 1
    elif kind == "granite":
        H, P, N = hf["mamba_n_heads"], hf["mamba_d_head"], hf["mamba_d_state"]
        G = hf.get("mamba_n_groups", 1)
        lim = hf.get("time_step_limit") or [0.001, 100.0]
        cfg.linear_kind = "mamba2"
        cfg.linear_num_key_heads, cfg.linear_key_head_dim = G, N
        cfg.linear_num_value_heads, cfg.linear_value_head_dim = H, P
        cfg.linear_conv_kernel_dim = hf.get("mamba_d_conv", 4)
        cfg.mamba_norm_group = (H * P) // G
        cfg.mamba_conv_bias = hf.get("mamba_conv_bias", True)
        cfg.ssm_dt_limits = (float(lim[0]), float(lim[-1]))
        cfg.layer_types = ["mamba" if t == "mamba" else "full_attention" for t in hf["layer_types"]]
        cfg.layer_blocks = None  # mixer + FFN in every layer
        cfg.layer_windows = None
        if hf.get("position_embedding_type", "rope") == "nope":
            cfg.partial_rotary_factor = 0.0
        cfg.extra["mamba_proj_bias"] = hf.get("mamba_proj_bias", False)
        if hf.get("num_local_experts"):
            cfg.num_experts = hf["num_local_experts"]
            cfg.moe_intermediate_size = hf["intermediate_size"]
            cfg.router_mode = "topk_softmax"
            cfg.moe_layers = None
            cfg.shared_expert_intermediate_size = hf.get("shared_intermediate_size", 0)
            cfg.shared_expert_gate = False
        else:
            cfg.num_experts = 0
        cfg.extra.update(residual_multiplier=hf.get("residual_multiplier", 1.0),
                         logits_scaling=hf.get("logits_scaling", 1.0))
        cfg.embed_scale = hf.get("embedding_multiplier", 1.0)
        if hf.get("attention_multiplier"):
            cfg.attn_scale = hf["attention_multiplier"]
        return
    else:
        H, P, N = hf["mamba_num_heads"], hf["mamba_head_dim"], hf["ssm_state_size"]
        pat = hf.get("hybrid_override_pattern")
        if isinstance(pat, list):
            pat = "".join(pat)
        if not pat and hf.get("layers_block_type"):
            pat = "".join(_NEMOTRON_BLOCKS[b] for b in hf["layers_block_type"])
        if not pat or len(pat) != cfg.num_layers:
            raise ValueError("nemotron_h needs hybrid_override_pattern or layers_block_type of num_hidden_layers")
        if "E" in pat:
            raise NotImplementedError("NemotronH MoE (E) layers are not served")
        pattern = pat
        norm_groups = hf.get("n_groups", 1)
    G = hf.get("n_groups", 1)
    cfg.linear_kind = "mamba2"
    cfg.linear_num_key_heads, cfg.linear_key_head_dim = G, N
    cfg.linear_num_value_heads, cfg.linear_value_head_dim = H, P
    cfg.linear_conv_kernel_dim = hf.get("conv_kernel", 4)
    cfg.mamba_norm_group = (H * P) // norm_groups
    cfg.mamba_conv_bias = hf.get("use_conv_bias", True)
    cfg.ssm_dt_limits = _ssm_dt_limits(hf)
    cfg.layer_types = [{"M": "mamba", "*": "full_attention", "-": "mlp"}[c] for c in pattern]
    cfg.layer_blocks = ["ffn" if c == "-" else "mixer" for c in pattern]
    cfg.layer_windows = None
    cfg.partial_rotary_factor = 0.0  # NemotronH attention has no positional rotation
    cfg.hidden_act = "relu2"
    cfg.mlp_bias = hf.get("mlp_bias", False)
    cfg.attention_bias = hf.get("attention_bias", False)
    cfg.extra["mamba_proj_bias"] = hf.get("mamba_proj_bias", hf.get("use_bias", False))
register("cohere", cohere=True)  # Command-R: LayerNorm, parallel attention + SwiGLU, logit scale
register("starcoder2", starcoder2=True)  # LayerNorm with bias, biased GELU MLP (c_fc / c_proj)


def supported_model_types() -> list[str]:
    return sorted(FAMILIES)


def build_config(hf: dict) -> DecoderConfig:
    """Translate a HF / MLX config.json dict."""
    if "text_config" in hf and ("hidden_size" not in hf or hf.get("model_type") not in FAMILIES):
        hf = {**hf["text_config"], "model_type": hf["text_config"].get("model_type", hf.get("model_type"))}
    mt = hf.get("model_type", "llama")
    if mt in _REFUSED:
        raise NotImplementedError(f"model_type {mt!r} needs {_REFUSED[mt]}, which this framework does not serve yet")
    tr = FAMILIES.get(mt)
    if tr is None:
        raise ValueError(f"unsupported model_type {mt!r}; supported: {', '.join(supported_model_types())}")
    if tr.get("ssm"):
        hf = _ssm_prepare(hf, tr["ssm"])
    hidden = hf["hidden_size"]
    heads = hf["num_attention_heads"]
    kvh = hf.get("num_key_value_heads") or heads
    hd = hf.get("head_dim") or hidden // heads
    cfg = DecoderConfig(
        model_type=mt, vocab_size=hf["vocab_size"], hidden_size=hidden, num_layers=hf["num_hidden_layers"],
        num_heads=heads, num_kv_heads=kvh, head_dim=hd, intermediate_size=hf.get("intermediate_size", 0),
        rms_norm_eps=hf.get("rms_norm_eps", hf.get("layer_norm_eps", 1e-6)),
        rope_theta=hf.get("rope_theta", 10000.0), rope_scaling=hf.get("rope_scaling"),
        partial_rotary_factor=hf.get("partial_rotary_factor", 1.0),
        max_position_embeddings=hf.get("max_position_embeddings", 4096),
        tie_word_embeddings=hf.get("tie_word_embeddings", False), qk_norm=tr.get("qk_norm", False),
        attention_bias=hf.get("attention_bias", mt in ("qwen2", "qwen2_vl", "qwen2_5_vl", "mimo")),
        o_bias=hf.get("o_bias", False),
        mlp_bias=hf.get("mlp_bias", False), quantization=hf.get("quantization") or hf.get("quantization_config"),
        hidden_act=_act(hf.get("hidden_activation") or hf.get("hidden_act") or "silu"))
    if cfg.rope_scaling and cfg.rope_scaling.get("rope_type", cfg.rope_scaling.get("type")) == "default":
        cfg.rope_scaling = None
    sw = hf.get("sliding_window")
    layer_types = hf.get("layer_types")
    if layer_types:
        cfg.layer_windows = [int(sw or 0) if t == "sliding_attention" else 0 for t in layer_types]
    elif sw and hf.get("use_sliding_window", True) and mt in ("mistral", "qwen2") and hf.get("use_sliding_window", False):
        cfg.layer_windows = [int(sw)] * cfg.num_layers
    if tr.get("moe"):
        cfg.num_experts = hf.get("num_experts", hf.get("num_local_experts", 0))
        cfg.num_experts_per_tok = hf.get("num_experts_per_tok", 2)
        cfg.moe_intermediate_size = hf.get("moe_intermediate_size", cfg.intermediate_size)
        cfg.norm_topk_prob = hf.get("norm_topk_prob", mt in ("mixtral", "phimoe"))
        step = hf.get("decoder_sparse_step", 1)
        mlp_only = set(hf.get("mlp_only_layers", []) or [])
        cfg.moe_layers = [(i not in mlp_only) and ((i + 1) % step == 0) for i in range(cfg.num_layers)]
        cfg.shared_expert_intermediate_size = hf.get("shared_expert_intermediate_size", 0)
        cfg.shared_expert_gate = bool(cfg.shared_expert_intermediate_size)
    if tr.get("hybrid"):
        # Gated DeltaNet layers with gated full attention every
        # `full_attention_interval` layers (MLXLLM/Models/Qwen3Next.swift:452)
        cfg.linear_num_key_heads = hf.get("linear_num_key_heads", 16)
        cfg.linear_num_value_heads = hf.get("linear_num_value_heads", 32)
        cfg.linear_key_head_dim = hf.get("linear_key_head_dim", 128)
        cfg.linear_value_head_dim = hf.get("linear_value_head_dim", 128)
        cfg.linear_conv_kernel_dim = hf.get("linear_conv_kernel_dim", 4)
        if layer_types and all(t in ("linear_attention", "full_attention") for t in layer_types):
            cfg.layer_types = list(layer_types)
        else:
            k = hf.get("full_attention_interval", 4)
            cfg.layer_types = ["full_attention" if (i + 1) % k == 0 else "linear_attention"
                               for i in range(cfg.num_layers)]
        cfg.layer_windows = None
        cfg.attn_output_gate = hf.get("attn_output_gate", True)
    if tr.get("lfm2_moe") or tr.get("bailing"):
        cfg.num_experts = hf.get("num_experts", 0)
        cfg.num_experts_per_tok = hf.get("num_experts_per_tok", 2)
        cfg.moe_intermediate_size = hf.get("moe_intermediate_size", cfg.intermediate_size)
        cfg.norm_topk_prob = hf.get("norm_topk_prob", True)
        cfg.routed_scaling_factor = float(hf.get("routed_scaling_factor", 1.0))
        n_dense = hf.get("num_dense_layers", hf.get("first_k_dense_replace", 0))
        cfg.moe_layers = [i >= n_dense for i in range(cfg.num_layers)]
        sig = tr.get("lfm2_moe") or hf.get("score_function", "sigmoid") == "sigmoid" or \
            hf.get("moe_router_enable_expert_bias", False)
        cfg.router_mode = "sigmoid_group" if sig else "softmax_topk"
        cfg.router_n_group = hf.get("n_group", 1) or 1
        cfg.router_topk_group = hf.get("topk_group", 1) or 1
    if tr.get("lfm2_moe"):
        cfg.intermediate_size = hf.get("intermediate_size", cfg.intermediate_size)
        cfg.extra["lfm2_moe"] = True
    if tr.get("bailing"):
        ns = hf.get("num_shared_experts") or 0
        cfg.shared_expert_intermediate_size = (hf.get("moe_shared_expert_intermediate_size")
                                               or cfg.moe_intermediate_size) * ns if ns else 0
        cfg.qk_norm = bool(hf.get("use_qk_norm", False))
        cfg.attention_bias = bool(hf.get("use_qkv_bias", False))
        cfg.o_bias = bool(hf.get("use_bias", False))
        cfg.tie_word_embeddings = hf.get("tie_word_embeddings", False)
    if tr.get("apertus"):
        cfg.hidden_act = "xielu"
        cfg.extra["norm_names"] = ("attention_layernorm", "feedforward_layernorm")
    if tr.get("post_only_norms"):
        cfg.pre_norms = False
        cfg.post_norms = True
    if tr.get("qk_norm_full"):
        cfg.qk_norm_full = True
    if tr.get("exaone4"):
        pat = hf.get("sliding_window_pattern")
        if isinstance(pat, int):  # every pat-th layer global
            pat = "L" * (pat - 1) + "G"
        if pat:
            local = [pat[i % len(pat)] == "L" for i in range(cfg.num_layers)]
            cfg.layer_windows = [int(sw or 0) if lo else 0 for lo in local]
            cfg.nope_layers = [i for i, lo in enumerate(local) if not lo]
    if mt == "olmo3" and layer_types and cfg.rope_scaling:
        # sliding layers rotate with the plain base; full layers with the scaled table
        cfg.extra["rope_local_theta"] = cfg.rope_theta
    g = tr.get("gemma")
    if g:
        cfg.embed_scale = math.sqrt(hidden)
        cfg.norm_offset_one = True
        cfg.hidden_act = "gelu_tanh"
        qpas = hf.get("query_pre_attn_scalar")
        if qpas:
            cfg.attn_scale = qpas ** -0.5
        if g >= 2:
            cfg.post_norms = True
            cfg.attn_logit_softcap = hf.get("attn_logit_softcapping") or 0.0
            cfg.final_logit_softcap = hf.get("final_logit_softcapping") or 0.0
            if not layer_types and sw:
                if g == 2:
                    cfg.layer_windows = [int(sw) if i % 2 == 0 else 0 for i in range(cfg.num_layers)]
                else:
                    pat = hf.get("sliding_window_pattern", 6)
                    cfg.layer_windows = [0 if (i + 1) % pat == 0 else int(sw) for i in range(cfg.num_layers)]
        if g == 3:
            cfg.qk_norm = True
            cfg.extra["rope_local_theta"] = hf.get("rope_local_base_freq", 10000.0)
        cfg.tie_word_embeddings = hf.get("tie_word_embeddings", True)
    if tr.get("gpt_oss"):
        cfg.num_experts = hf.get("num_local_experts", 128)
        cfg.num_experts_per_tok = hf.get("num_experts_per_tok", hf.get("experts_per_token", 4))
        cfg.moe_intermediate_size = hf.get("intermediate_size")
        cfg.router_mode = "topk_softmax"
        cfg.router_bias = True
        cfg.attention_bias = True
        cfg.o_bias = True
        cfg.mlp_bias = True
        cfg.attention_sinks = True
        cfg.hidden_act = "swiglu_oai"
        cfg.extra["swiglu_limit"] = hf.get("swiglu_limit", 7.0)
        if not layer_types:
            cfg.layer_windows = [int(sw or 128) if i % 2 == 0 else 0 for i in range(cfg.num_layers)]
    rp = hf.get("rope_parameters") or {}
    if rp and isinstance(rp.get("full_attention"), dict) and not tr.get("gemma4"):
        # per-layer-type parameters (transformers 5 configs): full layers take the
        # main table, sliding layers their own base
        full, slide = rp["full_attention"], rp.get("sliding_attention") or {}
        if full.get("rope_theta") is not None:
            cfg.rope_theta = float(full["rope_theta"])
        if full.get("rope_type", "default") not in ("default", None) and cfg.rope_scaling is None:
            cfg.rope_scaling = dict(full)
        if slide.get("rope_theta") is not None and cfg.layer_windows:
            cfg.extra["rope_local_theta"] = float(slide["rope_theta"])
        rp = {}
    if rp:
        if "rope_theta" not in hf and rp.get("rope_theta") is not None:
            cfg.rope_theta = float(rp["rope_theta"])
        if cfg.rope_scaling is None and rp.get("rope_type", rp.get("type", "default")) != "default":
            cfg.rope_scaling = dict(rp)
        if rp.get("llama_4_scaling_beta") and rp.get("original_max_position_embeddings"):
            cfg.extra["attn_pos_scale"] = (float(rp["llama_4_scaling_beta"]),
                                           int(rp["original_max_position_embeddings"]))
    if tr.get("phi2"):
        # MLXLLM/Models/Phi.swift: LayerNorm (with bias) before a parallel
        # attention + GELU MLP block, biased projections, final LayerNorm,
        # biased head, rotary on partial_rotary_factor of the head
        cfg.norm_kind = "layernorm"
        cfg.parallel_block = True
        cfg.hidden_act = "gelu_tanh_mlp"
        cfg.attention_bias = cfg.o_bias = cfg.mlp_bias = True
        cfg.partial_rotary_factor = hf.get("partial_rotary_factor", 0.4)
        cfg.rms_norm_eps = hf.get("layer_norm_eps", 1e-5)
        cfg.tie_word_embeddings = hf.get("tie_word_embeddings", False)
    if tr.get("lfm2"):
        # gated short-conv layers + attention layers, SwiGLU w1/w3/w2 FFN with
        # the auto-adjusted width (MLXLLM/Models/LFM2.swift:36-110, 240-262)
        n = cfg.num_layers
        lt = hf.get("layer_types")
        full = hf.get("full_attn_idxs")
        if lt:
            kinds = ["full_attention" if t == "full_attention" else "conv" for t in lt]
        elif full is not None:
            kinds = ["full_attention" if i in set(full) else "conv" for i in range(n)]
        else:
            kinds = ["full_attention"] * n
        cfg.layer_types = kinds
        cfg.layer_windows = None
        cfg.linear_kind = "short_conv"
        cfg.linear_conv_kernel_dim = hf.get("conv_L_cache", 3)
        cfg.mamba_conv_bias = hf.get("conv_bias", False)
        ff = hf.get("block_ff_dim", hf.get("intermediate_size", 4 * hidden))
        if hf.get("block_auto_adjust_ff_dim", False):
            ff = int(2 * ff / 3)
            if hf.get("block_ffn_dim_multiplier"):
                ff = int(hf["block_ffn_dim_multiplier"] * ff)
            mo = hf.get("block_multiple_of", 256)
            ff = mo * ((ff + mo - 1) // mo)
        cfg.intermediate_size = ff
        cfg.rms_norm_eps = hf.get("norm_eps", cfg.rms_norm_eps)
        cfg.tie_word_embeddings = hf.get("tie_word_embeddings", True)
    if tr.get("deepseek_router"):
        # routed + shared experts after `first_k_dense_replace` dense layers,
        # sigmoid (or softmax) scores with group-limited corrected selection
        # (MLXLLM/Models/GLM4MOE.swift:115-240)
        cfg.num_experts = hf.get("n_routed_experts", 0)
        cfg.moe_layers = [i >= hf.get("first_k_dense_replace", 0) for i in range(cfg.num_layers)]
        cfg.norm_topk_prob = hf.get("norm_topk_prob", True)
        cfg.router_mode = "sigmoid_group" if hf.get("scoring_func", "sigmoid") == "sigmoid" else "softmax_topk"
        cfg.router_n_group = hf.get("n_group", 1) or 1
        cfg.router_topk_group = hf.get("topk_group", 1) or 1
        cfg.routed_scaling_factor = float(hf.get("routed_scaling_factor", 1.0))
        cfg.shared_expert_intermediate_size = cfg.moe_intermediate_size * (hf.get("n_shared_experts") or 0)
        cfg.shared_expert_gate = False
        cfg.qk_norm = hf.get("use_qk_norm", False)
        cfg.attention_bias = hf.get("attention_bias", False)
    if tr.get("mla"):
        from . import mla

        mla.config_from_hf(cfg, hf)
        if mt == "deepseek_v2":
            # softmax gate, greedy or group-limited greedy top-k, no renormalisation
            # (MLXLLM/Models/DeepseekV2.swift:252-274)
            if hf.get("scoring_func", "softmax") != "softmax":
                raise NotImplementedError(f"DeepSeek V2 scoring_func {hf.get('scoring_func')!r} is not served")
            cfg.norm_topk_prob = hf.get("norm_topk_prob", False)
            cfg.router_mode = "softmax_topk"
            if hf.get("topk_method", "greedy") != "group_limited_greedy":
                cfg.router_n_group = cfg.router_topk_group = 1
    if tr.get("gemma4"):
        from . import gemma4

        gemma4.config_from_hf(cfg, hf)
    if tr.get("ssm"):
        _ssm_config(cfg, hf, tr["ssm"])
    if tr.get("diffusion"):
        cfg.extra["mask_token_id"] = hf.get("mask_token_id", 100)
        cfg.extra["diffusion_block"] = hf.get("block_size", 32)
    cfg.extra["fused_qkv"] = tr.get("fused_qkv", False)
    cfg.extra["fused_gate_up"] = tr.get("fused_gate_up", False)
    cfg.extra["mixtral_names"] = tr.get("mixtral_names", False)
    if tr.get("cohere"):
        if hf.get("use_qk_norm"):
            raise NotImplementedError("Cohere per-head LayerNorm q/k norms are not served")
        cfg.norm_kind = "layernorm"
        cfg.parallel_block = True
        cfg.rms_norm_eps = hf.get("layer_norm_eps", 1e-5)
        cfg.tie_word_embeddings = hf.get("tie_word_embeddings", True)
        cfg.extra["logits_scaling"] = 1.0 / float(hf.get("logit_scale", 1.0))
    if tr.get("starcoder2"):
        cfg.norm_kind = "layernorm"
        cfg.rms_norm_eps = hf.get("norm_epsilon", hf.get("layer_norm_eps", 1e-5))
        cfg.attention_bias = cfg.o_bias = cfg.mlp_bias = hf.get("use_bias", True)
        cfg.hidden_act = "gelu_tanh_mlp"
        if sw:
            cfg.layer_windows = [int(sw)] * cfg.num_layers
    if mt == "hunyuan_v1_dense" and hf.get("use_qk_norm"):
        raise NotImplementedError("Hunyuan q/k norms after the rotation are not served")
    if mt == "minicpm":  # MLXLLM/Models/MiniCPM.swift:107-180
        cfg.embed_scale = hf.get("scale_emb", 1.0)
        cfg.extra.update(residual_multiplier=hf.get("scale_depth", 1.0) / math.sqrt(cfg.num_layers),
                         logits_scaling=cfg.hidden_size / hf.get("dim_model_base", cfg.hidden_size))
    if mt == "granite":
        cfg.extra.update(embedding_multiplier=hf.get("embedding_multiplier", 1.0),
                         residual_multiplier=hf.get("residual_multiplier", 1.0),
                         logits_scaling=hf.get("logits_scaling", 1.0))
        cfg.embed_scale = hf.get("embedding_multiplier", 1.0)
        if hf.get("attention_multiplier"):
            cfg.attn_scale = hf["attention_multiplier"]
    return cfg


def _act(a: str) -> str:
    a = a.lower()
    if a in ("gelu_pytorch_tanh", "gelu_tanh", "gelu_new", "gelu"):
        return "gelu_tanh"
    return "silu"
