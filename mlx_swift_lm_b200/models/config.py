"""Decoder configuration shared by every text model family.

The reference implements ~70 model families as separate Swift files
(MLXLLM/Models/*, registry MLXLLM/LLMModelFactory.swift:71-143). Almost all
of them are the same pre-norm decoder with a handful of switches (qk-norm,
projection biases, sliding-window layers, sinks, softcaps, sandwich norms,
MoE FFNs, tied heads, RoPE variants). Here one fused decoder
(:mod:`.decoder`) takes those switches from :class:`DecoderConfig`, and each
family is a small adapter (:mod:`.families`) that maps its ``config.json`` and
checkpoint names onto it.
"""
from __future__ import annotations

from dataclasses import dataclass, field, fields


@dataclass
class DecoderConfig:
    model_type: str = "qwen3"
    vocab_size: int = 4096
    hidden_size: int = 256
    num_layers: int = 4
    num_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 64
    intermediate_size: int = 768
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    rope_scaling: dict | None = None
    partial_rotary_factor: float = 1.0
    rope_interleaved: bool = False
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = False
    # attention switches
    qk_norm: bool = False
    attention_bias: bool = False  # q/k/v projection bias
    o_bias: bool = False
    layer_windows: list[int] | None = None  # per-layer sliding window (0 = full attention)
    attention_sinks: bool = False
    attn_logit_softcap: float = 0.0
    final_logit_softcap: float = 0.0
    attn_scale: float | None = None  # default head_dim ** -0.5
    # norm / embedding switches
    embed_scale: float = 1.0
    norm_offset_one: bool = False  # weight stored as (w - 1), applied as (1 + w) (Gemma)
    post_norms: bool = False  # sandwich norms around attention and FFN (Gemma 2/3)
    # False: no input norms before attention / FFN, only the post-sublayer norms (OLMo 2/3, EXAONE 4)
    pre_norms: bool = True
    # q/k RMSNorm over the whole projection (all heads; weights [H*D], [KVH*D]) instead of per head (OLMo 2/3)
    qk_norm_full: bool = False
    # layers that apply no rotary embedding (EXAONE 4's global layers)
    nope_layers: list[int] | None = None
    # FFN
    hidden_act: str = "silu"  # silu | gelu_tanh | swiglu_oai
    mlp_bias: bool = False
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    # softmax_topk (Qwen/Mixtral) | topk_softmax (GPT-OSS) | sigmoid_group (GLM-4.5 / DeepSeek-V3:
    # sigmoid scores, corrected selection within the best router_topk_group of router_n_group groups)
    router_mode: str = "softmax_topk"
    router_n_group: int = 1
    router_topk_group: int = 1
    routed_scaling_factor: float = 1.0
    router_bias: bool = False
    moe_layers: list[bool] | None = None
    shared_expert_intermediate_size: int = 0
    shared_expert_gate: bool = False
    # hybrid linear-attention layers (Gated DeltaNet: Qwen3-Next, Qwen 3.5 / 3.6)
    layer_types: list[str] | None = None  # per layer "full_attention" | "linear_attention"
    attn_output_gate: bool = False  # q_proj also yields a sigmoid gate on the attention output
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    # "gdn" (Gated DeltaNet) | "mamba2" (Mamba-2 mixers: key heads = n_groups,
    # key dim = ssm state size, value heads = SSM heads, value dim = head dim)
    linear_kind: str = "gdn"
    ssm_dt_limits: tuple = (0.0, float("inf"))
    mamba_norm_group: int = 0  # channels per group of the gated RMSNorm (0: one group)
    mamba_conv_bias: bool = True
    # "rmsnorm" | "layernorm" (with bias; Phi-2); parallel_block: x + attn(ln(x)) + mlp(ln(x))
    norm_kind: str = "rmsnorm"
    parallel_block: bool = False
    # per layer "both" (mixer + FFN), "mixer" (mixer only) or "ffn" (FFN only);
    # None = "both" everywhere (NemotronH / Mamba2 layers hold one block each)
    layer_blocks: list[str] | None = None
    # quantization of the checkpoint (MLX layout), informational
    quantization: dict | None = None
    # MTP (multi-token prediction) modules
    num_mtp_layers: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def scale(self) -> float:
        return self.attn_scale if self.attn_scale is not None else self.head_dim ** -0.5

    def window(self, layer: int) -> int:
        if not self.layer_windows:
            return 0
        return int(self.layer_windows[layer])

    def max_window(self) -> int:
        return max((int(w) for w in self.layer_windows or ()), default=0)

    def is_linear(self, layer: int) -> bool:
        return bool(self.layer_types) and self.layer_types[layer] in ("linear_attention", "mamba", "conv")

    def block(self, layer: int) -> str:
        return self.layer_blocks[layer] if self.layer_blocks else "both"

    def has_attention(self, layer: int) -> bool:
        return not self.is_linear(layer) and self.block(layer) != "ffn"

    @property
    def gdn_dims(self) -> tuple[int, int, int, int]:
        """(key heads, key head dim, value heads, value head dim) of the linear layers."""
        return (self.linear_num_key_heads, self.linear_key_head_dim, self.linear_num_value_heads,
                self.linear_value_head_dim)

    @property
    def gdn_conv_dim(self) -> int:
        if self.linear_kind == "short_conv":  # LFM2: the conv runs over Bx (hidden channels)
            return self.hidden_size
        Hk, Dk, Hv, Dv = self.gdn_dims
        return 2 * Hk * Dk + Hv * Dv

    @property
    def gdn_in_dim(self) -> int:
        """Rows of the fused linear-layer in-projection: q | k | v | z | b | a
        (Mamba-2: C | B | x | z | dt)."""
        if self.linear_kind == "short_conv":
            return 3 * self.hidden_size
        Hk, Dk, Hv, Dv = self.gdn_dims
        return self.gdn_conv_dim + Hv * Dv + (Hv if self.linear_kind == "mamba2" else 2 * Hv)

    def is_moe(self, layer: int) -> bool:
        if self.num_experts <= 0:
            return False
        if self.moe_layers is None:
            return True
        return bool(self.moe_layers[layer])

    @property
    def glu_epi(self) -> str:
        return {"silu": "swiglu", "gelu_tanh": "geglu", "gelu": "geglu", "swiglu_oai": "swiglu_oai",
                "relu2": "relu2", "gelu_tanh_mlp": "gelu_tanh", "xielu": "xielu"}[self.hidden_act]

    def to_dict(self) -> dict:
        return {f.name: getattr(self, f.name) for f in fields(self)}

    @classmethod
    def from_dict(cls, d: dict) -> "DecoderConfig":
        names = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in names})


# --- benchmark configurations -------------------------------------------------
def tiny_qwen3() -> DecoderConfig:
    """benchmark config 1: 4 layers, d 256, 4q/2kv, hd 64, SwiGLU 768, vocab 4096, tied."""
    return DecoderConfig(model_type="qwen3", vocab_size=4096, hidden_size=256, num_layers=4, num_heads=4,
                         num_kv_heads=2, head_dim=64, intermediate_size=768, rms_norm_eps=1e-6, rope_theta=1e6,
                         tie_word_embeddings=True, qk_norm=True, max_position_embeddings=4096)


def qwen3_8b() -> DecoderConfig:
    """benchmark config 2: Qwen3-8B shape."""
    return DecoderConfig(model_type="qwen3", vocab_size=151936, hidden_size=4096, num_layers=36, num_heads=32,
                         num_kv_heads=8, head_dim=128, intermediate_size=12288, rms_norm_eps=1e-6, rope_theta=1e6,
                         tie_word_embeddings=False, qk_norm=True, max_position_embeddings=40960)


def qwen3_30b_a3b() -> DecoderConfig:
    """benchmark config 3: Qwen3-30B-A3B shape (+1 MTP module)."""
    return DecoderConfig(model_type="qwen3_moe", vocab_size=151936, hidden_size=2048, num_layers=48, num_heads=32,
                         num_kv_heads=4, head_dim=128, intermediate_size=6144, rms_norm_eps=1e-6, rope_theta=1e6,
                         qk_norm=True, num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                         norm_topk_prob=True, max_position_embeddings=40960, num_mtp_layers=1)


def gpt_oss_120b() -> DecoderConfig:
    """benchmark config 4: GPT-OSS-120B shape."""
    return DecoderConfig(model_type="gpt_oss", vocab_size=201088, hidden_size=2880, num_layers=36, num_heads=64,
                         num_kv_heads=8, head_dim=64, intermediate_size=2880, rms_norm_eps=1e-5, rope_theta=150000,
                         rope_scaling={"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                       "original_max_position_embeddings": 4096, "truncate": False},
                         attention_bias=True, o_bias=True, layer_windows=[128 if i % 2 == 0 else 0 for i in range(36)],
                         attention_sinks=True, hidden_act="swiglu_oai", mlp_bias=True, num_experts=128,
                         num_experts_per_tok=4, moe_intermediate_size=2880, router_mode="topk_softmax",
                         router_bias=True, max_position_embeddings=131072)


def llama3_70b() -> DecoderConfig:
    """benchmark config 5: Llama-3-70B shape."""
    return DecoderConfig(model_type="llama", vocab_size=128256, hidden_size=8192, num_layers=80, num_heads=64,
                         num_kv_heads=8, head_dim=128, intermediate_size=28672, rms_norm_eps=1e-5, rope_theta=500000,
                         rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                       "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                         max_position_embeddings=131072)
