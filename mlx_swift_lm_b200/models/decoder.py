"""The fused pre-norm decoder used by every text family.

Per layer (paged path, the serving hot path):

    h      = add_rmsnorm(x, delta)            # residual add + norm, one kernel
    qkv    = gemm(h, Wqkv)                    # tcgen05 GEMM (+ bias)
    q      = qk_norm_rope_kv(qkv, ...)        # qk-norm + RoPE + paged K/V append
    attn   = paged_decode(q[:Bd]) | paged_prefill(q[Bd:])
    delta  = gemm(attn, Wo)                   # (+ tensor-parallel reduction)
    h      = add_rmsnorm(x, delta)
    delta  = gemm(gemm(h, Wgate_up, epi=glu), Wdown)   or the MoE block

Parity: MLXLLM/Models/Qwen3.swift:56-216 (attention, block, model), Llama.swift,
GPTOSS.swift:122-381 (sinks, alternating windows), Qwen3MoE.swift:114-156 (MoE);
the ``LanguageModel`` protocol surface (MLXLMCommon/LanguageModel.swift:331-463)
is :class:`DecoderLM`'s ``new_cache`` / ``forward_dense`` / ``forward``.
"""
from __future__ import annotations

import math
import os

import torch

from .. import ops
from ..ops import reference as ref
from ..ops.qlinear import QuantizedWeight
from .batch import ForwardBatch
from .config import DecoderConfig
from .rope import build_rope


class LayerWeights:
    __slots__ = ("ln1", "wqkv", "bqkv", "q_norm", "k_norm", "wo", "bo", "ln2", "post_attn_norm", "post_ffn_norm",
                 "wgu", "bgu", "wd", "bd", "router", "router_b", "experts_gu", "experts_gu_b", "experts_d",
                 "experts_d_b", "shared_gu", "shared_d", "shared_gate", "sinks", "moe",
                 # sigmoid_group routers: the selection-score correction (e_score_correction_bias)
                 "router_corr",
                 # linear-attention (Gated DeltaNet) layers: wqkv is the fused in-projection
                 # q|k|v|z|b|a and wo the out-projection
                 "linear", "conv_w", "A_log", "dt_bias", "gdn_norm",
                 # Mamba-2 mixers (same fused layout; conv bias and the D skip term)
                 "conv_b", "ssm_D",
                 # "both" | "mixer" | "ffn": which blocks the layer holds
                 "block",
                 # LayerNorm biases of the input / post-attention norms (norm_kind "layernorm")
                 "ln1_b", "ln2_b",
                 # ParoQuant: activation rotations shared by the experts (gate/up input, down input)
                 "experts_rot_in", "experts_rot_mid",
                 # xIELU MLP activation: raw (alpha_p, alpha_n, beta, eps) of the layer (Apertus)
                 "act_params",
                 # multi-head latent attention (DeepSeek V2 / V3): query LoRA down / norm / up, the
                 # joint latent + shared rotary-key projection, its norm, and the per-head k_nope | v up
                 "mla_q_a", "mla_q_a_norm", "mla_q_b", "mla_kv_a", "mla_kv_a_norm", "mla_kv_b",
                 # Gemma 4: router input scale and per-expert weight scales, the dense / expert branch
                 # norms of the MoE block, the per-layer-input gate / projection / norm, the layer scalar
                 "g4_router_scale", "g4_expert_scale", "g4_post_ffn1", "g4_pre_ffn2", "g4_post_ffn2",
                 "ple_gate", "ple_proj", "ple_norm", "layer_scalar")

    F32 = ("sinks", "conv_w", "A_log", "dt_bias", "conv_b", "ssm_D", "router_corr", "act_params", "layer_scalar")  # kept in fp32 whatever the model dtype

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)

    def tensors(self):
        for s in self.__slots__:
            v = getattr(self, s)
            if isinstance(v, torch.Tensor):
                yield s, v
            elif hasattr(v, "tensors"):
                for n, t in v.tensors():
                    yield f"{s}.{n}", t


class TensorParallel:
    """Tensor-parallel context of a rank: which heads / channels / vocab rows
    it owns, and the reduction used after the row-parallel projections.
    With world == 1 every hook is the identity."""

    def __init__(self, rank: int = 0, world: int = 1, group=None, reducer=None):
        self.rank, self.world, self.group = rank, world, group
        self.reducer = reducer  # callable(t) -> reduced tensor (in place allowed)

    def reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        if self.reducer is not None:
            return self.reducer(t)
        import torch.distributed as dist

        dist.all_reduce(t, group=self.group)
        return t


class DenseKVCache:
    """Per-layer contiguous K/V grown by concatenation (the legacy
    KVCacheSimple of MLXLMCommon/KVCache.swift:470). CPU / reference path."""

    def __init__(self, num_layers: int):
        self.k = [None] * num_layers
        self.v = [None] * num_layers
        self.offset = 0

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        if self.k[layer] is None:
            self.k[layer], self.v[layer] = k, v
        else:
            self.k[layer] = torch.cat([self.k[layer], k], 0)
            self.v[layer] = torch.cat([self.v[layer], v], 0)
        return self.k[layer], self.v[layer]

    def rec_state(self, layer: int, model):
        """(conv, delta-rule) state of a linear-attention layer, one slot."""
        if not hasattr(self, "_rec"):
            self._rec = {}
        if layer not in self._rec:
            cfg = model.cfg
            Hk, Dk, Hv, Dv = cfg.gdn_dims
            dev, dt = model.device, model.dtype
            self._rec[layer] = (torch.zeros(1, cfg.linear_conv_kernel_dim - 1, cfg.gdn_conv_dim, dtype=dt, device=dev),
                                torch.zeros(1, Hv, Dv, Dk, dtype=torch.float32, device=dev))
        return self._rec[layer]

    def trim(self, n: int):
        """Drop the last n tokens (speculative rollback)."""
        n = min(n, self.offset)
        for i in range(len(self.k)):
            if self.k[i] is not None:
                self.k[i] = self.k[i][: self.k[i].shape[0] - n]
                self.v[i] = self.v[i][: self.v[i].shape[0] - n]
        self.offset -= n
        return n


class DecoderLM:
    """A decoder-only language model with paged-KV and dense-KV forwards."""

    # the paged forward routes each KV layer's slots and page tables through ForwardBatch.tables
    supports_window_ring = True

    def __new__(cls, cfg: DecoderConfig, *args, **kwargs):
        # families whose layers differ in attention geometry have their own subclass
        if cls is DecoderLM and cfg.extra.get("gemma4"):
            from .gemma4 import Gemma4LM

            cls = Gemma4LM
        return super().__new__(cls)

    def __init__(self, cfg: DecoderConfig, device="cpu", dtype=torch.float32, tp: TensorParallel | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.tp = tp or TensorParallel()
        w = self.tp.world
        assert cfg.num_heads % w == 0, "query heads must divide across TP ranks"
        self.H = cfg.num_heads // w
        self.KVH = max(1, cfg.num_kv_heads // w) if cfg.num_kv_heads >= w else 1
        self.D = cfg.head_dim
        self.F = cfg.intermediate_size // w if cfg.intermediate_size else 0
        self.Fe = cfg.moe_intermediate_size // w if cfg.moe_intermediate_size else 0
        self.embed = None
        self.norm = None
        self.norm_b = None  # final LayerNorm bias (norm_kind "layernorm")
        self.lm_head_b = None  # head bias (Phi-2)
        self.lm_head = None
        self.layers: list[LayerWeights] = []
        self.mtp_layers: list = []
        self.cos_sin, self.rot_dim = build_rope(cfg.head_dim, cfg.rope_theta, cfg.rope_scaling,
                                                cfg.max_position_embeddings, cfg.partial_rotary_factor)
        self.cos_sin = self.cos_sin.to(self.device)
        # sliding-window layers with their own rotary base (Gemma 3 local layers, OLMo 3 sliding layers)
        self.cos_sin_local = None
        lt = cfg.extra.get("rope_local_theta")
        if lt is not None:
            self.cos_sin_local, _ = build_rope(cfg.head_dim, float(lt), None, cfg.max_position_embeddings,
                                               cfg.partial_rotary_factor)
            self.cos_sin_local = self.cos_sin_local.to(self.device)
        self._nope = set(cfg.nope_layers or ())
        self.lora = None  # adapter whose update is currently added into the weights (adapters.lora)
        self.batched_lora = None  # adapters.batched.BatchedLoRA: per-row adapters, base weights untouched
        self._lora_slots = None  # per-token adapter slots of the forward in progress
        # hook(li, x, delta) -> (x, delta) after layer li of a forward (Qwen3-VL deepstack rows)
        self._after_layer = None
        self.tp_fused = None  # fused symmetric-memory TP decode path (parallel.tp_fused)
        # hybrid models: attention layers index the KV slab, linear layers the recurrent-state pool
        self.kv_index, self.rec_index = [], []
        na = nl = 0
        for li in range(cfg.num_layers):
            if cfg.is_linear(li):
                assert w == 1, "linear-attention layers run without tensor parallelism"
                self.kv_index.append(-1)
                self.rec_index.append(nl)
                nl += 1
            elif cfg.block(li) == "ffn":
                self.kv_index.append(-1)
                self.rec_index.append(-1)
            else:
                self.kv_index.append(na)
                self.rec_index.append(-1)
                na += 1
        self.num_kv_layers = na

    # ------------------------------------------------------------------ weights
    def named_tensors(self):
        yield "embed", self.embed
        yield "norm", self.norm
        if self.lm_head is not None and self.lm_head is not self.embed:
            yield "lm_head", self.lm_head
        for i, L in enumerate(self.layers):
            for n, t in L.tensors():
                yield f"layers.{i}.{n}", t

    def num_params(self) -> int:
        return sum(t.numel() for _, t in self.named_tensors() if t is not None)

    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True,
                    keep_layers: tuple[int, int] | None = None, layer_hook=None):
        """Random N(0, std) weights (norm weights 1, sinks N(0,1)), generated on
        the model's device. Every rank draws the full tensors from the same
        seed and keeps its tensor-parallel shard, so a TP=N model computes the
        same function as the TP=1 model of that seed. With `keep_layers`
        (lo, hi) every layer is still drawn (the generator advances exactly
        as for the full model) but only layers lo..hi-1 are kept: a pipeline
        stage of the same function. `layer_hook(L)` runs on each kept layer
        as soon as it is drawn (quantising the experts of a model whose bf16
        weights would not fit on the device at once)."""
        cfg = self.cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        dev, dt = self.device, self.dtype
        r, w = self.tp.rank, self.tp.world
        D = self.D

        def rn(*shape):
            t = torch.empty(shape, device=dev, dtype=dt)
            t.normal_(0.0, std, generator=g)
            return t

        def ones(n):
            return torch.zeros(n, device=dev, dtype=dt) if cfg.norm_offset_one else torch.ones(n, device=dev, dtype=dt)

        def rows(t, n_per):  # contiguous row block of this rank
            return t if w == 1 else t[r * n_per:(r + 1) * n_per].contiguous()

        def cols(t):
            if w == 1:
                return t
            n = t.shape[-1] // w
            return t[..., r * n:(r + 1) * n].contiguous()

        def kv_rows(t):
            if w == 1:
                return t
            if cfg.num_kv_heads >= w:
                return rows(t, self.KVH * D)
            h = (r * cfg.num_kv_heads) // w
            return t[h * D:(h + 1) * D].contiguous()

        def glu_pair(F_full, F_local, K, lead=()):
            gate, up = rn(*lead, F_full, K), rn(*lead, F_full, K)
            if lead:
                return torch.stack([ref.interleave_gate_up(rows(gate[e], F_local), rows(up[e], F_local))
                                    for e in range(lead[0])])
            return ref.interleave_gate_up(rows(gate, F_local), rows(up, F_local))

        hd = cfg.hidden_size
        if with_embeddings:
            self.embed = rn(cfg.vocab_size, hd)
            self.lm_head = self.embed if cfg.tie_word_embeddings else rn(cfg.vocab_size, hd)
        self.norm = ones(hd)
        self.layers = []
        for li in range(cfg.num_layers):
            L = LayerWeights()
            L.ln1 = ones(hd)
            L.ln2 = ones(hd)
            L.linear = cfg.is_linear(li)
            L.block = cfg.block(li)
            if L.block == "ffn":  # FFN-only layer: ln1 is its norm
                L.ln2 = None
                self._init_ffn(L, li, rn, ones, rows, cols, glu_pair)
                if keep_layers is None or keep_layers[0] <= li < keep_layers[1]:
                    self.layers.append(L if layer_hook is None else layer_hook(L) or L)
                continue
            if L.linear:
                self._init_linear_layer(L, rn, g)
                if L.block == "both":
                    self._init_ffn(L, li, rn, ones, rows, cols, glu_pair)
                else:
                    L.ln2 = None
                if keep_layers is None or keep_layers[0] <= li < keep_layers[1]:
                    self.layers.append(L if layer_hook is None else layer_hook(L) or L)
                continue
            if cfg.extra.get("mla"):
                from . import mla

                assert w == 1, "multi-head latent attention loads without tensor parallelism"
                mla.init_random(self, L, rn, ones)
                if cfg.post_norms:
                    L.post_attn_norm = ones(hd)
                    L.post_ffn_norm = ones(hd)
                if L.block == "both":
                    self._init_ffn(L, li, rn, ones, rows, cols, glu_pair)
                if keep_layers is None or keep_layers[0] <= li < keep_layers[1]:
                    self.layers.append(L if layer_hook is None else layer_hook(L) or L)
                continue
            wq, wk, wv = rn(cfg.q_size, hd), rn(cfg.kv_size, hd), rn(cfg.kv_size, hd)
            L.wqkv = torch.cat([rows(wq, self.H * D), kv_rows(wk), kv_rows(wv)], 0)
            if cfg.attn_output_gate:  # gate rows after q|k|v: the attention kernels read q|k|v only
                L.wqkv = torch.cat([L.wqkv, rows(rn(cfg.q_size, hd), self.H * D)], 0)
            if cfg.attention_bias:
                bq, bk, bv = rn(cfg.q_size), rn(cfg.kv_size), rn(cfg.kv_size)
                L.bqkv = torch.cat([rows(bq, self.H * D), kv_rows(bk), kv_rows(bv)], 0)
            if cfg.qk_norm_full:
                L.q_norm = ones(self.H * D)
                L.k_norm = ones(self.KVH * D)
            elif cfg.qk_norm:
                L.q_norm = ones(D)
                L.k_norm = ones(D)
            L.wo = cols(rn(hd, cfg.q_size))
            if cfg.o_bias:
                bo = rn(hd)
                L.bo = bo if r == 0 else torch.zeros_like(bo)
            if cfg.post_norms:
                L.post_attn_norm = ones(hd)
                L.post_ffn_norm = ones(hd)
            if cfg.attention_sinks:
                s = torch.empty(cfg.num_heads, device=dev, dtype=torch.float32).normal_(0.0, 1.0, generator=g)
                L.sinks = rows(s, self.H)
            if L.block == "both":
                self._init_ffn(L, li, rn, ones, rows, cols, glu_pair)
            else:
                L.ln2 = None
            if not cfg.pre_norms:  # post-sublayer norms only
                L.ln1 = L.ln2 = None
                L.post_attn_norm = ones(hd)
                L.post_ffn_norm = ones(hd)
            if keep_layers is None or keep_layers[0] <= li < keep_layers[1]:
                self.layers.append(L if layer_hook is None else layer_hook(L) or L)
        return self

    def _init_ffn(self, L, li, rn, ones, rows, cols, glu_pair):
        cfg = self.cfg
        r, w = self.tp.rank, self.tp.world
        hd = cfg.hidden_size
        if cfg.is_moe(li):
            E = cfg.num_experts
            Fe = cfg.moe_intermediate_size
            L.moe = True
            L.router = rn(E, hd)
            if cfg.router_bias:
                L.router_b = rn(E)
            if cfg.router_mode == "sigmoid_group":
                L.router_corr = rn(E).float()
            L.experts_gu = glu_pair(Fe, self.Fe, hd, (E,))
            L.experts_d = cols(rn(E, hd, Fe))
            if cfg.mlp_bias:
                gb, ub = rn(E, Fe), rn(E, Fe)
                L.experts_gu_b = torch.stack([ref.interleave_gate_up(rows(gb[e], self.Fe)[:, None],
                                                                     rows(ub[e], self.Fe)[:, None])[:, 0]
                                              for e in range(E)])
                db = rn(E, hd)
                L.experts_d_b = db if r == 0 else torch.zeros_like(db)
            if cfg.shared_expert_intermediate_size:
                Fs = cfg.shared_expert_intermediate_size
                L.shared_gu = glu_pair(Fs, Fs // w, hd)
                L.shared_d = cols(rn(hd, Fs))
                if cfg.shared_expert_gate:
                    L.shared_gate = rn(1, hd)
        else:
            L.moe = False
            F = cfg.intermediate_size
            if cfg.glu_epi in ("relu2", "gelu_tanh", "xielu"):  # non-gated MLP: wgu holds the up projection only
                L.wgu = rows(rn(F, hd), self.F)
                L.wd = cols(rn(hd, F))
                if cfg.glu_epi == "xielu":
                    L.act_params = torch.tensor([0.55, 0.55, 0.5, -1e-6], dtype=torch.float32, device=self.device)
                return
            L.wgu = glu_pair(F, self.F, hd)
            L.wd = cols(rn(hd, F))
            if cfg.mlp_bias:
                gb, ub = rn(F), rn(F)
                L.bgu = ref.interleave_gate_up(rows(gb, self.F)[:, None], rows(ub, self.F)[:, None])[:, 0]
                bd = rn(hd)
                L.bd = bd if r == 0 else torch.zeros_like(bd)

    def _init_linear_layer(self, L, rn, g):
        """Gated DeltaNet weights: fused in-projection q|k|v|z|b|a, depthwise
        conv taps, decay parameters (A_log = log U(1, 16), dt_bias = 1),
        gated-norm weight, out-projection."""
        cfg = self.cfg
        hd = cfg.hidden_size
        Hk, Dk, Hv, Dv = cfg.gdn_dims
        C = cfg.gdn_conv_dim
        dev = self.device
        L.wqkv = rn(cfg.gdn_in_dim, hd)
        L.conv_w = rn(C, cfg.linear_conv_kernel_dim).float()
        L.A_log = torch.empty(Hv, device=dev, dtype=torch.float32).uniform_(1.0, 16.0, generator=g).log_()
        L.dt_bias = torch.ones(Hv, device=dev, dtype=torch.float32)
        if cfg.linear_kind == "short_conv":  # LFM2: in_proj B|C|x, depthwise conv taps (+ bias), out_proj
            L.conv_b = rn(C).float() if cfg.mamba_conv_bias else None
            L.A_log = L.dt_bias = None
            L.wo = rn(hd, hd)
            return
        if cfg.linear_kind == "mamba2":  # gated group norm over all channels; conv bias; D skip
            L.gdn_norm = torch.ones(Hv * Dv, device=dev, dtype=self.dtype)
            L.conv_b = rn(C).float() if cfg.mamba_conv_bias else None
            L.ssm_D = torch.ones(Hv, device=dev, dtype=torch.float32)
        else:
            L.gdn_norm = torch.ones(Dv, device=dev, dtype=self.dtype)
        L.wo = rn(hd, Hv * Dv)

    # ------------------------------------------------------------------ pieces
    def _attn_out(self, L, attn2d):
        delta = ops.gemm(attn2d, L.wo, bias=L.bo if self.tp.rank == 0 or L.bo is None else None)
        lo = self._lora(L, "o")
        if lo is not None:
            self._lora_add(lo, attn2d, delta)
        return self.tp.reduce(delta)

    def _mlp(self, L, h):
        cfg = self.cfg
        if L.moe:
            return self._moe(L, h)
        lo = self._lora(L, "gu")
        if lo is not None and cfg.glu_epi in ("swiglu", "geglu", "swiglu_oai"):
            from ..ops import lora as lops

            pre = ops.gemm(h, L.wgu, bias=L.bgu)
            slots, A, Bt, scale = lo
            t = lops.lora_shrink(h, A, slots, out=self.batched_lora.scratch(h.shape[0], A.shape[1], h.device))
            gu = lops.lora_expand_glu(pre, Bt, t, slots, scale, cfg.glu_epi)
        elif lo is not None:
            raise NotImplementedError(f"batched LoRA on a {cfg.glu_epi!r} MLP")
        elif cfg.glu_epi == "xielu":
            gu = ops.xielu(ops.gemm(h, L.wgu, bias=L.bgu), L.act_params)
        else:
            gu = ops.gemm(h, L.wgu, epi=cfg.glu_epi, bias=L.bgu)
        delta = ops.gemm(gu, L.wd, bias=L.bd if self.tp.rank == 0 else None)
        lo = self._lora(L, "d")
        if lo is not None:
            self._lora_add(lo, gu, delta)
        return self.tp.reduce(delta)

    def route(self, L, h):
        """Router top-k: returns (weights [T, k] fp32, ids [T, k] expert ids)."""
        cfg = self.cfg
        from ..ops import moe as moe_ops

        logits = ops.gemm(h, L.router, epi="f32", bias=L.router_b)
        w, idx = moe_ops.route_topk(logits, cfg.num_experts_per_tok, cfg.router_mode, cfg.norm_topk_prob,
                                    L.router_corr, cfg.router_n_group, cfg.router_topk_group,
                                    cfg.routed_scaling_factor)
        return w.float(), idx

    def _moe(self, L, h):
        from ..ops import moe as moe_ops

        cfg = self.cfg
        w, idx = self.route(L, h)
        out = moe_ops.moe_experts(h, L.experts_gu, L.experts_d, w, idx, cfg.glu_epi, L.experts_gu_b,
                                  L.experts_d_b if self.tp.rank == 0 else None, rot_in=L.experts_rot_in,
                                  rot_mid=L.experts_rot_mid)
        if L.shared_gu is not None:
            s = ops.gemm(ops.gemm(h, L.shared_gu, epi=cfg.glu_epi), L.shared_d)
            if L.shared_gate is not None:
                s = (torch.sigmoid(ops.gemm(h, L.shared_gate, epi="f32")) * s.float()).to(s.dtype)
            out = (out.float() + s.float()).to(out.dtype)
        return self.tp.reduce(out)

    def _final_logits(self, h):
        logits = ops.gemm(h, self.lm_head, epi="f32", bias=self.lm_head_b)
        if self.cfg.final_logit_softcap > 0:
            c = self.cfg.final_logit_softcap
            logits = torch.tanh(logits / c) * c
        return logits

    # ------------------------------------------------------------------ paged forward
    def _lora(self, L, target):
        """(slots, A, B^T, scale) of the batched adapters of this layer's
        projection when the forward in progress has adapter rows, else None."""
        bl, slots = self.batched_lora, self._lora_slots
        if bl is None or slots is None:
            return None
        ab = bl.tensors(L, target)
        return None if ab is None else (slots, ab[0], ab[1], bl.scale)

    def _lora_add(self, lo, x, y):
        """y += per-row adapter delta of input x (in place)."""
        from ..ops import lora as lops

        slots, A, Bt, scale = lo
        t = lops.lora_shrink(x, A, slots, out=self.batched_lora.scratch(x.shape[0], A.shape[1], x.device))
        return lops.lora_expand(y, Bt, t, slots, scale)

    def forward(self, fb: ForwardBatch, kv, return_hidden: bool = False, inputs_embeds: torch.Tensor | None = None,
                return_both: bool = False, return_residual: bool = False):
        """Paged-KV forward over a flattened batch. Returns fp32 logits for
        ``fb.logit_idx`` rows (all tokens when None); with `return_hidden` the
        final-normed hidden rows instead, with `return_both` (logits, hidden).
        `inputs_embeds` [T, H] replaces the token embedding (MTP modules,
        pipeline stages after the first); `return_residual` returns the
        residual stream of every token after the last layer instead (pipeline
        stages before the last)."""
        self._lora_slots = fb.lora_slots if self.batched_lora is not None else None
        try:
            with ops.row_roles(fb.num_tokens, fb.num_decode):
                return self._forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        finally:
            self._lora_slots = None

    def _forward(self, fb, kv, return_hidden, inputs_embeds, return_both, return_residual):
        cfg = self.cfg
        T = fb.num_tokens
        nd = fb.num_decode
        x = inputs_embeds if inputs_embeds is not None else ops.embedding(fb.input_ids, self.embed, cfg.embed_scale)
        delta = None
        attn = torch.empty((T, self.H, self.D), dtype=x.dtype, device=x.device)
        hook = self._after_layer
        for li, L in enumerate(self.layers):
            if hook is not None and li > 0:
                x, delta = hook(li - 1, x, delta)
            h = self._norm(x, delta, L.ln1, L.ln1_b)
            if L.block == "ffn":  # FFN-only layer (NemotronH "-" / "E")
                delta = self._mlp(L, h)
                continue
            if cfg.parallel_block:  # Phi-2: attention and MLP read the same normed input
                a = self._attention(L, h, fb, kv, li, attn)
                delta = (a.float() + self._mlp(L, h).float()).to(x.dtype)
                continue
            if L.linear:
                delta = self._gdn(L, h, fb, kv, li)
            else:
                delta = self._attention(L, h, fb, kv, li, attn)
            if L.post_attn_norm is not None:
                delta = ops.rmsnorm(delta, L.post_attn_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
            if L.block == "mixer":
                continue
            h = self._norm(x, delta, L.ln2, L.ln2_b)
            delta = self._mlp(L, h)
            if L.post_ffn_norm is not None:
                delta = ops.rmsnorm(delta, L.post_ffn_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
        return self._head(x, delta, fb, return_hidden, return_both, return_residual)

    def _attention(self, L, h, fb: ForwardBatch, kv, li: int, attn: torch.Tensor) -> torch.Tensor:
        """Paged attention of one layer (decode rows, then prefill chunks);
        returns the output projection (before the residual add)."""
        if L.mla_kv_a is not None:
            from . import mla

            return mla.attention(self, L, h, fb, kv, li, attn)
        cfg = self.cfg
        T, nd = fb.num_tokens, fb.num_decode
        ki = self.kv_index[li] if self.kv_index else li
        kc, vc = kv.layer(ki)
        cos_sin, rot_dim = self.rope_for(li)
        positions = fb.positions
        if fb.rope_table is not None:  # per-token rotary rows (M-RoPE prompts)
            cos_sin = fb.rope_table
            positions = torch.arange(T, dtype=torch.int32, device=fb.positions.device)
        qkv = None
        slots, dec_pt, pf_pt = fb.tables(kv, ki)
        lo = self._lora(L, "qkv")
        if lo is None and self._fused_qkv_rope(L, h, fb, rot_dim):
            q = ops.gemm_qkv_rope(h, L.wqkv, L.bqkv, positions, slots, cos_sin, L.q_norm, L.k_norm,
                                  cfg.rms_norm_eps, kc, vc, self.H, self.KVH, kv.k_scale(ki), kv.v_scale(ki))
        else:
            qkv = ops.gemm(h, L.wqkv, bias=L.bqkv)
            if lo is not None:
                self._lora_add(lo, h, qkv)
            qn, kn = L.q_norm, L.k_norm
            if cfg.qk_norm_full:
                qkv = self._qk_full_norm(L, qkv)
                qn = kn = None
            q = ops.qk_norm_rope_kv(qkv, positions, slots, cos_sin, rot_dim, cfg.rope_interleaved,
                                    qn, kn, cfg.rms_norm_eps, kc, vc, self.H, self.KVH, self.D,
                                    kv.k_scale(ki), kv.v_scale(ki))
        q = self._pos_scale_q(q, fb.positions)
        win = cfg.window(li)
        if nd:
            ops.paged_decode(q[:nd], kc, vc, dec_pt, fb.dec_seq_lens, cfg.scale, win, L.sinks,
                             cfg.attn_logit_softcap, kv.k_scale(ki), kv.v_scale(ki), fb.dec_max_parts,
                             out=attn[:nd])
        if T > nd:
            ops.paged_prefill(q[nd:], kc, vc, pf_pt, fb.pf_cu_q, fb.pf_pos0, cfg.scale,
                              -1 if fb.bidirectional else win, L.sinks,
                              cfg.attn_logit_softcap, kv.k_scale(ki), kv.v_scale(ki), fb.pf_cu_q_host,
                              out=attn[nd:])
        a2 = attn.view(T, self.H * self.D)
        if cfg.attn_output_gate:
            from ..ops.gdn import sigmoid_mul

            g0 = (self.H + 2 * self.KVH) * self.D
            a2 = sigmoid_mul(a2, qkv[:, g0:g0 + self.H * self.D])
        return self._attn_out(L, a2)

    # class switch: qkv GEMM with the qk-norm / RoPE / KV append epilogue where it applies
    fused_qkv_rope = os.environ.get("B200LM_FUSED_QKV_ROPE", "1") != "0"

    def rope_for(self, li: int):
        """(cos|sin table, rotary dims) of layer li: the local table for
        sliding-window layers when the model has one, none for NoPE layers."""
        if li in self._nope:
            return self.cos_sin, 0
        if self.cos_sin_local is not None and self.cfg.window(li) > 0:
            return self.cos_sin_local, self.rot_dim
        return self.cos_sin, self.rot_dim

    def _fused_qkv_rope(self, L, h, fb, rot_dim) -> bool:
        """The fused epilogue covers head dim 128 with full non-interleaved
        rotary from the position table, bf16 weights, no output gate rows."""
        cfg = self.cfg
        return (self.fused_qkv_rope and h.is_cuda and self.D == 128 and rot_dim == 128
                and not cfg.rope_interleaved and not cfg.attn_output_gate and not cfg.qk_norm_full
                and fb.rope_table is None and isinstance(L.wqkv, torch.Tensor) and L.wqkv.dtype == torch.bfloat16
                and self.cos_sin.shape[-1] == 128)

    def _qk_full_norm(self, L, qkv):
        """RMSNorm over the whole q and k projections (all heads), in place."""
        cfg = self.cfg
        H, KVH, D = self.H, self.KVH, self.D
        q = ops.rmsnorm(qkv[:, :H * D].contiguous(), L.q_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
        k = ops.rmsnorm(qkv[:, H * D:(H + KVH) * D].contiguous(), L.k_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
        qkv[:, :H * D] = q
        qkv[:, H * D:(H + KVH) * D] = k
        return qkv

    def _norm(self, x, delta, w, b=None):
        """x <- x + delta; the block's input norm (RMSNorm, or LayerNorm with bias).
        Blocks without input norms (OLMo 2/3, EXAONE 4) get the residual stream itself."""
        cfg = self.cfg
        if w is None and not cfg.pre_norms:
            if delta is not None:
                x.add_(delta)
            return x
        if cfg.norm_kind == "layernorm":
            return ops.add_layernorm(x, delta, w, b, cfg.rms_norm_eps)
        return ops.add_rmsnorm(x, delta, w, cfg.rms_norm_eps, offset_one=cfg.norm_offset_one)

    def _pos_scale_q(self, q, positions):
        """Llama-4 query scaling by position (Ministral 3 / Nemotron-Labs-
        Diffusion ``llama_4_scaling_beta``): q * (1 + beta * log(1 +
        floor(p / original_max_position_embeddings)))."""
        ps = self.cfg.extra.get("attn_pos_scale")
        if not ps:
            return q
        beta, orig = ps
        s = 1.0 + beta * torch.log1p(torch.floor(positions.float() / orig))
        return (q.float() * s[:, None, None]).to(q.dtype)

    def _gdn_rows(self, fb: ForwardBatch):
        """Rows of `fb` for the linear-attention layers (cached on the batch):
        decode rows are one token each and never fresh; a prefill chunk is
        fresh when it starts at position 0."""
        from ..ops.gdn import GdnRows

        rows = getattr(fb, "_gdn_rows", None)
        if rows is not None:
            return rows
        dev = fb.input_ids.device
        nd = fb.num_decode
        assert fb.state_slots is not None, "hybrid models need the rows' recurrent-state slots"
        if fb.num_tokens == nd:  # pure decode: device-side construction (graph-capturable)
            cu = torch.arange(nd + 1, dtype=torch.int32, device=dev)
            fresh = torch.zeros(nd, dtype=torch.int32, device=dev)
            cu_host = None
        else:
            pf = fb.pf_cu_q_host or [0]
            cu_host = list(range(nd + 1)) + [nd + c for c in pf[1:]]
            cu = torch.tensor(cu_host, dtype=torch.int32).to(dev)
            fresh = torch.cat([torch.zeros(nd, dtype=torch.int32, device=dev), (fb.pf_pos0 == 0).to(torch.int32)])
        rows = GdnRows(cu, fresh, fb.state_slots.to(torch.int32), cu_host)
        fb._gdn_rows = rows
        return rows

    def _gdn(self, L, h, fb: ForwardBatch, kv, li: int) -> torch.Tensor:
        from ..ops.gdn import gdn_layer

        cfg = self.cfg
        P = ops.gemm(h, L.wqkv, bias=L.bqkv)
        conv, ssm = kv.rec.layer(self.rec_index[li])
        return self._attn_out(L, self._linear_body(L, P, self._gdn_rows(fb), conv, ssm))

    def _linear_body(self, L, P, rows, conv, ssm):
        """Gated DeltaNet or Mamba-2 body on the fused in-projection P."""
        from ..ops.gdn import gdn_layer, mamba_layer

        cfg = self.cfg
        Hk, Dk, Hv, Dv = cfg.gdn_dims
        if cfg.linear_kind == "short_conv":
            from ..ops.gdn import short_conv

            return short_conv(P, rows, conv, L.conv_w, L.conv_b)
        if cfg.linear_kind == "mamba2":
            grp = cfg.mamba_norm_group or Hv * Dv
            return mamba_layer(P, rows, conv, ssm, L.conv_w, L.conv_b, L.A_log, L.dt_bias, L.ssm_D, L.gdn_norm, Hk,
                               Dk, Hv, Dv, cfg.rms_norm_eps, grp, cfg.ssm_dt_limits)
        return gdn_layer(P, rows, conv, ssm, L.conv_w, L.A_log, L.dt_bias, L.gdn_norm, Hk, Dk, Hv, Dv,
                         cfg.rms_norm_eps)

    def _head(self, x, delta, fb, return_hidden, return_both, return_residual):
        cfg = self.cfg
        if return_residual:
            return (x.float() + delta.float()).to(x.dtype) if delta is not None else x
        if fb.logit_idx is not None:
            xs = (x.float() + delta.float()).to(x.dtype)[fb.logit_idx] if delta is not None else x[fb.logit_idx]
            if cfg.norm_kind == "layernorm":
                h = ops.add_layernorm(xs.contiguous(), None, self.norm, self.norm_b, cfg.rms_norm_eps)
            else:
                h = ops.rmsnorm(xs.contiguous(), self.norm, cfg.rms_norm_eps, cfg.norm_offset_one)
        elif cfg.norm_kind == "layernorm":
            h = ops.add_layernorm(x, delta, self.norm, self.norm_b, cfg.rms_norm_eps)
        else:
            h = ops.add_rmsnorm(x, delta, self.norm, cfg.rms_norm_eps, offset_one=cfg.norm_offset_one)
        if return_hidden:
            return h
        if return_both:
            return self._final_logits(h), h
        return self._final_logits(h)

    # ------------------------------------------------------------------ decode step -> tokens
    def enable_fused_tp(self, max_rows: int):
        """Use the fused symmetric-memory collectives for decode steps of up
        to `max_rows` rows (tensor parallel only)."""
        if self.tp.world > 1:
            if any(isinstance(t, QuantizedWeight) for L in self.layers for t in (L.wqkv, L.wo, L.wgu, L.wd)):
                raise ValueError("the fused TP decode path serves bf16 weights; quantised models use NCCL TP")
            from ..parallel.tp_fused import FusedTP

            self.tp_fused = FusedTP(self, max_rows)
        return self

    def begin_step(self):
        """Advance the collective step counter (every rank, once per decode step)."""
        if getattr(self, "tp_fused", None) is not None:
            self.tp_fused.comm.begin_step()

    def forward_greedy_both(self, fb: ForwardBatch, kv):
        """(greedy token [rows] int32, final hidden [rows, H]) of the logit
        rows: the batched verify of speculative decoding needs no more."""
        logits, h = self.forward(fb, kv, return_both=True)
        return ops.argmax(logits), h

    def forward_decode_tokens(self, fb: ForwardBatch, kv, out: torch.Tensor, out2=None, flags=None):
        """Greedy tokens of a pure-decode batch: the fused TP path when
        enabled, else forward + argmax. `flags` (int32 [rows]) receives the
        non-finite-logit flag of each row (the fused TP path's split argmax
        leaves it untouched)."""
        tpf = getattr(self, "tp_fused", None)
        if tpf is not None and fb.num_decode == fb.num_tokens and fb.num_tokens <= tpf.M_pad:
            return tpf.decode_tokens(fb, kv, out, out2)
        logits = self.forward(fb, kv)
        return ops.argmax(logits, out=out, out2=out2, flags=flags)

    # ------------------------------------------------------------------ dense forward
    def new_cache(self) -> DenseKVCache:
        return DenseKVCache(self.cfg.num_layers)

    @torch.no_grad()
    def forward_dense(self, tokens: torch.Tensor, cache: DenseKVCache, return_hidden: bool = False,
                      bidirectional: bool = False):
        """Single-sequence forward with a dense, concatenating KV cache (the
        legacy single-request path). tokens [L] int; returns logits [L, V].
        `bidirectional`: the new tokens attend to each other both ways (and
        to the whole cache), as mask-diffusion blocks do."""
        cfg = self.cfg
        Lq = tokens.shape[0]
        p0 = cache.offset
        positions = torch.arange(p0, p0 + Lq, dtype=torch.int32, device=tokens.device)
        x = ops.embedding(tokens.to(torch.int32), self.embed, cfg.embed_scale)
        delta = None
        for li, L in enumerate(self.layers):
            h = self._norm(x, delta, L.ln1, L.ln1_b)
            if L.block == "ffn":
                delta = self._mlp(L, h)
                continue
            if L.linear:
                from ..ops.gdn import GdnRows

                conv, ssm = cache.rec_state(li, self)
                i32 = dict(dtype=torch.int32, device=x.device)
                rows = GdnRows(torch.tensor([0, Lq], **i32), torch.tensor([1 if p0 == 0 else 0], **i32),
                               torch.zeros(1, **i32), [0, Lq])
                delta = self._attn_out(L, self._linear_body(L, ops.gemm(h, L.wqkv, bias=L.bqkv), rows, conv, ssm))
            elif L.mla_kv_a is not None:
                from . import mla

                delta = mla.dense_attention(self, L, h, cache, li, positions)
            else:
                qkv = ops.gemm(h, L.wqkv, bias=L.bqkv)
                qn, kn = L.q_norm, L.k_norm
                if cfg.qk_norm_full:
                    qkv = self._qk_full_norm(L, qkv)
                    qn = kn = None
                cs, rd = self.rope_for(li)
                q, k, v = ops.qk_norm_rope_kv(qkv, positions, None, cs, rd, cfg.rope_interleaved,
                                              qn, kn, cfg.rms_norm_eps, None, None, self.H, self.KVH,
                                              self.D, return_kv=True)
                ki = self.kv_index[li] if self.kv_index else li
                kk, vv = cache.update(ki, k, v)
                kpos = cache.key_positions(ki) if hasattr(cache, "key_positions") else None
                extra = cache.chunk_mask if hasattr(cache, "chunk_mask") else None
                q = self._pos_scale_q(q, positions)
                a = ref.attention_rows_ref(q.float(), kk.float(), vv.float(), positions, kk.shape[0], cfg.scale,
                                           -1 if bidirectional else cfg.window(li), L.sinks, cfg.attn_logit_softcap,
                                           k_pos=kpos, extra_mask=extra).to(x.dtype)
                a2 = a.reshape(Lq, self.H * self.D).contiguous()
                if cfg.attn_output_gate:
                    from ..ops.gdn import sigmoid_mul

                    g0 = (self.H + 2 * self.KVH) * self.D
                    a2 = sigmoid_mul(a2, qkv[:, g0:g0 + self.H * self.D])
                delta = self._attn_out(L, a2)
            if cfg.parallel_block:
                delta = (delta.float() + self._mlp(L, h).float()).to(x.dtype)
                continue
            if L.post_attn_norm is not None:
                delta = ops.rmsnorm(delta, L.post_attn_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
            if L.block == "mixer":
                continue
            h = self._norm(x, delta, L.ln2, L.ln2_b)
            delta = self._mlp(L, h)
            if L.post_ffn_norm is not None:
                delta = ops.rmsnorm(delta, L.post_ffn_norm, cfg.rms_norm_eps, cfg.norm_offset_one)
        cache.offset += Lq
        h = self._norm(x, delta, self.norm, self.norm_b)
        if return_hidden:
            return h
        return self._final_logits(h)

    # ------------------------------------------------------------------ misc
    def clone_to(self, device, dtype) -> "DecoderLM":
        """A copy of this model (weights converted) on another device / dtype."""
        m = DecoderLM(self.cfg, device, dtype, tp=self.tp)
        dev = torch.device(device)

        def cv(t, keep_f32=False):
            if t is None:
                return None
            return t.to(device=dev, dtype=torch.float32 if keep_f32 else dtype)

        m.embed = cv(self.embed)
        m.norm = cv(self.norm)
        m.norm_b = cv(self.norm_b)
        m.lm_head_b = cv(self.lm_head_b)
        if self.lm_head is self.embed:
            m.lm_head = m.embed
        elif isinstance(self.lm_head, QuantizedWeight):
            m.lm_head = self.lm_head.to(dev)
        else:
            m.lm_head = cv(self.lm_head)
        for L in self.layers:
            N = LayerWeights()
            for s in LayerWeights.__slots__:
                v = getattr(L, s)
                if isinstance(v, torch.Tensor):
                    v = cv(v, s in LayerWeights.F32)
                elif isinstance(v, QuantizedWeight):
                    v = v.to(dev)
                elif v is not None and hasattr(v, "to") and not isinstance(v, bool):  # rotated weights, rotations
                    v = v.to(dev, dtype)
                setattr(N, s, v)
            m.layers.append(N)
        return m

    def kv_layer_geom(self) -> list[tuple[int, int, int]]:
        """(KV heads, head dim, window) of every layer that owns paged KV, in
        KV-slab order."""
        cfg = self.cfg
        return [(self.KVH, self.D, cfg.window(li)) for li in range(cfg.num_layers)
                if not self.kv_index or self.kv_index[li] >= 0]

    def attn_scratch_dims(self) -> tuple[int, int]:
        """(query heads, head dim) bounding every attention layer's split-KV scratch."""
        return self.H, self.D

    def kv_bytes_per_token(self, kv_dtype=None) -> int:
        dt = kv_dtype or self.dtype
        es = torch.empty((), dtype=dt).element_size()
        return sum(2 * kvh * d * es for kvh, d, _ in self.kv_layer_geom())

    def to(self, device=None, dtype=None):
        device = torch.device(device) if device is not None else self.device
        dtype = dtype or self.dtype

        def mv(t):
            if t is None:
                return None
            if not isinstance(t, torch.Tensor):  # quantised / rotated weights
                return t.to(device, dtype) if not isinstance(t, QuantizedWeight) else t.to(device)
            if t.is_floating_point() and t.dtype != torch.float32 or (t.dtype == torch.float32 and dtype != torch.float32):
                return t.to(device=device, dtype=dtype if t.dtype != torch.float32 or True else t.dtype)
            return t.to(device=device)

        tied = self.lm_head is self.embed
        self.embed = mv(self.embed)
        self.norm = mv(self.norm)
        self.norm_b = mv(self.norm_b)
        self.lm_head_b = mv(self.lm_head_b)
        self.lm_head = self.embed if tied else mv(self.lm_head)
        for L in self.layers:
            for s in LayerWeights.__slots__:
                v = getattr(L, s)
                if v is not None and not isinstance(v, (torch.Tensor, bool)) and hasattr(v, "to"):
                    setattr(L, s, v.to(device, dtype))
                    continue
                if isinstance(v, torch.Tensor):
                    if s in LayerWeights.F32:
                        setattr(L, s, v.to(device=device, dtype=torch.float32))
                    else:
                        setattr(L, s, v.to(device=device, dtype=dtype))
        self.cos_sin = self.cos_sin.to(device)
        if self.cos_sin_local is not None:
            self.cos_sin_local = self.cos_sin_local.to(device)
        self.device, self.dtype = device, dtype
        return self


def softmax_scale(cfg: DecoderConfig) -> float:
    return cfg.scale if cfg.attn_scale is not None else 1.0 / math.sqrt(cfg.head_dim)
