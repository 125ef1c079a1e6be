"""Gemma 4 text models (gemma4 / gemma4_text: E2B / E4B dense with per-layer
inputs, 26B-A4B mixture of experts, 31B dense).

Structure (MLXLLM/Models/Gemma4Text.swift:795-1670):

* layer kinds from ``layer_types``: sliding layers (window ``sliding_window``,
  head dim ``head_dim``, ``num_key_value_heads``, default RoPE of
  ``rope_parameters.sliding_attention``) and full layers (head dim
  ``global_head_dim``, ``num_global_key_value_heads`` when given,
  proportional RoPE of ``rope_parameters.full_attention`` over the whole head
  with only ``partial_rotary_factor`` of the pairs rotated);
* attention scale 1; RMSNorm on q and k (learned scale) and on v (no scale);
  full layers with ``attention_k_eq_v`` take v from the raw (pre-norm) k;
* the last ``num_kv_shared_layers`` layers compute no K/V: each reads the
  cache of the last earlier layer of its kind (Gemma4TextModelInner
  previousKvs); their MLP is twice as wide with ``use_double_wide_mlp``;
* block: x += post_attn_norm(attn(input_norm(x))); then the GeGLU MLP on
  pre_ffn_norm(x) - with the MoE block, post_ffn_norm_1(mlp) plus
  post_ffn_norm_2(experts(pre_ffn_norm_2(x))) routed by a softmax-over-top-k
  router on rmsnorm(x) * scale / sqrt(hidden) with per-expert scales -
  through post_ffn_norm into the residual; then the per-layer input gate
  (E2B / E4B): x += norm(proj(gelu(gate(x)) * ple_i)); finally x *= layer_scalar;
* per-layer inputs: embed_tokens_per_layer(ids) * sqrt(ple_dim) plus
  norm(per_layer_model_projection(h0) / sqrt(hidden)), both [L, ple_dim] per
  token, summed and scaled by 2^-1/2;
* embeddings scaled by sqrt(hidden); final logits soft-capped.

The paged cache holds one slab per attention geometry (sliding and full
layers differ in KV heads and head dim), co-indexed by page; KV-shared layers
own no slab rows and read their source layer's.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..ops import reference as ref
from .config import DecoderConfig
from .decoder import DecoderLM, LayerWeights, TensorParallel
from .rope import build_rope


def g4(cfg: DecoderConfig) -> dict:
    return cfg.extra["gemma4"]


def config_from_hf(cfg: DecoderConfig, hf: dict):
    """Gemma 4 switches of a config.json (text_config already unwrapped)."""
    L = cfg.num_layers
    sw = int(hf.get("sliding_window") or 512)
    lt = hf.get("layer_types")
    if not lt:
        pat = int(hf.get("sliding_window_pattern") or 5)
        lt = ["full_attention" if (i % pat) == pat - 1 else "sliding_attention" for i in range(L)]
    lt = list(lt)[:L] + ["sliding_attention"] * max(0, L - len(lt))
    rp = hf.get("rope_parameters") or {}
    sl, fu = rp.get("sliding_attention") or {}, rp.get("full_attention") or {}
    n_shared = int(hf.get("num_kv_shared_layers") or 0)
    if hf.get("use_bidirectional_attention") == "all":
        raise NotImplementedError("Gemma 4 bidirectional (encoder) attention is not served by the causal engine")
    cfg.layer_windows = [sw if t == "sliding_attention" else 0 for t in lt]
    cfg.layer_types = None
    cfg.attn_scale = 1.0
    cfg.hidden_act = "gelu_tanh"
    cfg.embed_scale = math.sqrt(cfg.hidden_size)
    cfg.final_logit_softcap = float(hf.get("final_logit_softcapping") or 0.0)
    cfg.tie_word_embeddings = hf.get("tie_word_embeddings", True)
    cfg.qk_norm = True
    cfg.post_norms = True
    cfg.norm_offset_one = False
    cfg.rope_theta = float(sl.get("rope_theta", 10000.0))
    cfg.rope_scaling = None
    cfg.partial_rotary_factor = 1.0
    moe = bool(hf.get("enable_moe_block", False))
    if moe:
        cfg.num_experts = int(hf["num_experts"])
        cfg.num_experts_per_tok = int(hf.get("top_k_experts") or hf.get("num_experts_per_tok"))
        cfg.moe_intermediate_size = int(hf.get("moe_intermediate_size") or cfg.intermediate_size)
        cfg.router_mode = "topk_softmax"
        cfg.moe_layers = [False] * L  # the expert block is part of every layer's FFN, handled here
    gkv = hf.get("num_global_key_value_heads")
    cfg.extra["gemma4"] = dict(
        layer_types=lt, window=sw, global_head_dim=int(hf.get("global_head_dim") or cfg.head_dim),
        global_kv_heads=int(gkv) if gkv else cfg.num_kv_heads, k_eq_v=bool(hf.get("attention_k_eq_v", False)),
        kv_shared=n_shared, ple_dim=int(hf.get("hidden_size_per_layer_input") or 0),
        ple_vocab=int(hf.get("vocab_size_per_layer_input") or cfg.vocab_size),
        double_wide=bool(hf.get("use_double_wide_mlp", False)), moe=moe,
        full_theta=float(fu.get("rope_theta", 1_000_000.0)),
        full_rotary=float(fu.get("partial_rotary_factor", 1.0)), full_factor=float(fu.get("factor", 1.0)))


def proportional_rope(head_dim: int, base: float, rotary: float, factor: float, max_pos: int) -> torch.Tensor:
    """cos|sin table [max_pos, head_dim] of proportional RoPE: pairs (i,
    i + D/2) for every i < D/2; the first int(rotary * D / 2) rotate at
    1 / (factor * base^(2i/D)), the rest stay fixed (cos 1, sin 0)
    (MLXLMCommon/RoPEUtils.swift:164-230)."""
    n = int(rotary * head_dim / 2)
    inv = torch.zeros(head_dim // 2, dtype=torch.float64)
    if n:
        inv[:n] = 1.0 / (factor * base ** (torch.arange(0, 2 * n, 2, dtype=torch.float64) / head_dim))
    return ref.rope_cos_sin(inv, max_pos, 1.0)


class Gemma4LM(DecoderLM):
    """Gemma 4 text model on the paged engine (see the module docstring)."""

    def __init__(self, cfg: DecoderConfig, device="cpu", dtype=torch.float32, tp: TensorParallel | None = None):
        super().__init__(cfg, device, dtype, tp)
        if self.tp.world != 1:
            raise NotImplementedError("Gemma 4 loads without tensor parallelism")
        p = g4(cfg)
        Lc = cfg.num_layers
        self.kinds = ["full" if t == "full_attention" else "sliding" for t in p["layer_types"]]
        self.Dg, self.KVHg = p["global_head_dim"], p["global_kv_heads"]
        first_shared = Lc - p["kv_shared"] if p["kv_shared"] > 0 else Lc
        self.first_shared = first_shared
        # KV ownership: layers before the shared block own their K/V; shared
        # layers read the last earlier owner of their kind
        self.kv_index, self.rec_index = [], [-1] * Lc
        last = {}
        n = 0
        for li in range(Lc):
            if li < first_shared:
                self.kv_index.append(n)
                last[self.kinds[li]] = n
                n += 1
            else:
                src = last.get(self.kinds[li])
                if src is None:
                    raise ValueError(f"Gemma 4 layer {li} shares K/V but no earlier {self.kinds[li]} layer owns any")
                self.kv_index.append(src)
        self.num_kv_layers = n
        self.kv_owner = [li < first_shared for li in range(Lc)]
        mp = cfg.max_position_embeddings
        self.rope_s = self.cos_sin  # built by DecoderLM over head_dim with the sliding base
        self.rope_f = proportional_rope(self.Dg, p["full_theta"], p["full_rotary"], p["full_factor"], mp).to(self.device)
        self.ple_dim = p["ple_dim"]
        self.embed_ple = None  # [ple_vocab, L * ple_dim]
        self.ple_proj = None  # [L * ple_dim, hidden]
        self.ple_proj_norm = None  # [ple_dim]

    # ------------------------------------------------------------------ geometry
    def geom(self, li: int):
        """(KV heads, head dim, window) of layer li."""
        if self.kinds[li] == "full":
            return self.KVHg, self.Dg, 0
        return self.KVH, self.D, self.cfg.window(li)

    def kv_layer_geom(self):
        return [self.geom(li) for li in range(self.cfg.num_layers) if self.kv_owner[li]]

    def attn_scratch_dims(self):
        return self.H, max(self.D, self.Dg)

    def ffn_width(self, li: int) -> int:
        p = g4(self.cfg)
        return self.cfg.intermediate_size * (2 if p["double_wide"] and li >= self.first_shared else 1)

    def named_tensors(self):
        yield from super().named_tensors()
        for n in ("embed_ple", "ple_proj", "ple_proj_norm"):
            yield n, getattr(self, n)

    # ------------------------------------------------------------------ weights
    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True, keep_layers=None):
        cfg = self.cfg
        p = g4(cfg)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        dev, dt = self.device, self.dtype
        hd = cfg.hidden_size

        def rn(*shape):
            t = torch.empty(shape, device=dev, dtype=dt)
            t.normal_(0.0, std, generator=g)
            return t

        def ones(n):
            return torch.ones(n, device=dev, dtype=dt)

        if with_embeddings:
            self.embed = rn(cfg.vocab_size, hd)
            self.lm_head = self.embed if cfg.tie_word_embeddings else rn(cfg.vocab_size, hd)
        self.norm = ones(hd)
        if self.ple_dim:
            P, Lc = self.ple_dim, cfg.num_layers
            self.embed_ple = rn(p["ple_vocab"], Lc * P)
            self.ple_proj = rn(Lc * P, hd)
            self.ple_proj_norm = ones(P)
        self.layers = []
        for li in range(cfg.num_layers):
            L = LayerWeights()
            kvh, D, _ = self.geom(li)
            H = self.H
            L.ln1, L.post_attn_norm, L.ln2, L.post_ffn_norm = ones(hd), ones(hd), ones(hd), ones(hd)
            own = self.kv_owner[li]
            kv_rows = 0 if not own else (1 if p["k_eq_v"] and self.kinds[li] == "full" else 2) * kvh * D
            L.wqkv = rn(H * D + kv_rows, hd)
            L.q_norm = ones(D)
            L.k_norm = ones(D) if own else None
            L.wo = rn(hd, H * D)
            F = self.ffn_width(li)
            L.wgu = ref.interleave_gate_up(rn(F, hd), rn(F, hd))
            L.wd = rn(hd, F)
            if p["moe"]:
                E, Fe = cfg.num_experts, cfg.moe_intermediate_size
                L.router = rn(E, hd)
                L.g4_router_scale = ones(hd)
                L.g4_expert_scale = ones(E)
                L.experts_gu = torch.stack([ref.interleave_gate_up(rn(Fe, hd), rn(Fe, hd)) for _ in range(E)])
                L.experts_d = rn(E, hd, Fe)
                L.g4_post_ffn1, L.g4_pre_ffn2, L.g4_post_ffn2 = ones(hd), ones(hd), ones(hd)
            if self.ple_dim:
                L.ple_gate = rn(self.ple_dim, hd)
                L.ple_proj = rn(hd, self.ple_dim)
                L.ple_norm = ones(hd)
            L.layer_scalar = torch.ones(1, device=dev, dtype=torch.float32)
            self.layers.append(L)
        return self

    # ------------------------------------------------------------------ shared pieces
    def _ple_inputs(self, ids, x0):
        """Per-layer inputs [T, L, ple_dim] of the tokens `ids` with scaled embeddings x0."""
        cfg = self.cfg
        P, Lc = self.ple_dim, cfg.num_layers
        T = ids.shape[0]
        tok = ops.embedding(ids.to(torch.int32), self.embed_ple, math.sqrt(P)).view(T, Lc, P)
        proj = ops.gemm(x0, self.ple_proj, epi="f32") * (cfg.hidden_size ** -0.5)
        proj = ops.rmsnorm(proj.to(x0.dtype).reshape(T * Lc, P).contiguous(), self.ple_proj_norm,
                           cfg.rms_norm_eps).view(T, Lc, P)
        return ((proj.float() + tok.float()) * (2.0 ** -0.5)).to(x0.dtype)

    def _route(self, L, x):
        cfg = self.cfg
        from ..ops import moe as moe_ops

        ones = torch.ones_like(L.g4_router_scale)
        hn = ops.rmsnorm(x, ones, cfg.rms_norm_eps)
        hn = (hn.float() * L.g4_router_scale.float() * cfg.hidden_size ** -0.5).to(x.dtype)
        logits = ops.gemm(hn, L.router, epi="f32")
        w, idx = moe_ops.route_topk(logits, cfg.num_experts_per_tok, "topk_softmax", True)
        w = w.float() * L.g4_expert_scale.float()[idx.long()]
        return w, idx

    def _ffn(self, L, x):
        """The layer's feed-forward delta (before post_ffn_norm) for residual x."""
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        h = ops.rmsnorm(x, L.ln2, eps)
        m = ops.gemm(ops.gemm(h, L.wgu, epi=cfg.glu_epi), L.wd)
        if L.router is None:
            return m
        from ..ops import moe as moe_ops

        m1 = ops.rmsnorm(m, L.g4_post_ffn1, eps)
        w, idx = self._route(L, x)
        h2 = ops.rmsnorm(x, L.g4_pre_ffn2, eps)
        e = moe_ops.moe_experts(h2, L.experts_gu, L.experts_d, w, idx, cfg.glu_epi)
        m2 = ops.rmsnorm(e, L.g4_post_ffn2, eps)
        return (m1.float() + m2.float()).to(x.dtype)

    def _block_tail(self, L, li, x, attn_out, ple):
        """Everything after attention: residual adds, FFN, per-layer input, scalar."""
        eps = self.cfg.rms_norm_eps
        x = (x.float() + ops.rmsnorm(attn_out, L.post_attn_norm, eps).float()).to(x.dtype)
        x = (x.float() + ops.rmsnorm(self._ffn(L, x), L.post_ffn_norm, eps).float()).to(x.dtype)
        if ple is not None:
            gt = ops.gemm(x, L.ple_gate, epi="gelu_tanh")
            gt = (gt.float() * ple[:, li].float()).to(x.dtype)
            x = (x.float() + ops.rmsnorm(ops.gemm(gt, L.ple_proj), L.ple_norm, eps).float()).to(x.dtype)
        return (x.float() * L.layer_scalar.float()).to(x.dtype)

    def _qkv_parts(self, L, li, h):
        """(packed q|k|v for the norm/rope/append op, own-KV flag): v_norm is
        applied here; k_eq_v layers take v from the raw k; shared layers get
        zero k/v columns that are never written."""
        p = g4(self.cfg)
        kvh, D, _ = self.geom(li)
        H, T = self.H, h.shape[0]
        y = ops.gemm(h, L.wqkv)
        if not self.kv_owner[li]:
            z = torch.zeros(T, 2 * kvh * D, dtype=y.dtype, device=y.device)
            return torch.cat([y, z], 1)
        k = y[:, H * D:H * D + kvh * D]
        v = k if (p["k_eq_v"] and self.kinds[li] == "full") else y[:, H * D + kvh * D:H * D + 2 * kvh * D]
        ones = torch.ones(D, dtype=y.dtype, device=y.device)
        vn = ops.rmsnorm(v.reshape(T * kvh, D).contiguous(), ones, self.cfg.rms_norm_eps).view(T, kvh * D)
        return torch.cat([y[:, :H * D + kvh * D], vn], 1)

    def _rope(self, li):
        return (self.rope_f, self.Dg) if self.kinds[li] == "full" else (self.rope_s, self.D)

    # ------------------------------------------------------------------ paged forward
    def _forward(self, fb, kv, return_hidden, inputs_embeds, return_both, return_residual):
        cfg = self.cfg
        T, nd = fb.num_tokens, fb.num_decode
        x = inputs_embeds if inputs_embeds is not None else ops.embedding(fb.input_ids, self.embed, cfg.embed_scale)
        ple = self._ple_inputs(fb.input_ids, x) if self.ple_dim else None
        bufs = {}
        for li, L in enumerate(self.layers):
            kvh, D, win = self.geom(li)
            H = self.H
            h = ops.rmsnorm(x, L.ln1, cfg.rms_norm_eps)
            packed = self._qkv_parts(L, li, h)
            ki = self.kv_index[li]
            kc, vc = kv.layer(ki)
            cs, rd = self._rope(li)
            slots, dec_pt, pf_pt = fb.tables(kv, ki)
            if not self.kv_owner[li]:
                slots = torch.full_like(slots, -1)
            q = ops.qk_norm_rope_kv(packed, fb.positions, slots, cs, rd, False, L.q_norm, L.k_norm,
                                    cfg.rms_norm_eps, kc, vc, H, kvh, D, kv.k_scale(ki), kv.v_scale(ki))
            if D not in bufs:
                bufs[D] = torch.empty((T, H, D), dtype=x.dtype, device=x.device)
            attn = bufs[D]
            if nd:
                ops.paged_decode(q[:nd], kc, vc, dec_pt, fb.dec_seq_lens, cfg.scale, win, None, 0.0,
                                 kv.k_scale(ki), kv.v_scale(ki), fb.dec_max_parts, out=attn[:nd])
            if T > nd:
                ops.paged_prefill(q[nd:], kc, vc, pf_pt, fb.pf_cu_q, fb.pf_pos0, cfg.scale, win, None,
                                  0.0, kv.k_scale(ki), kv.v_scale(ki), fb.pf_cu_q_host, out=attn[nd:])
            a = ops.gemm(attn.view(T, H * D), L.wo)
            x = self._block_tail(L, li, x, a, ple)
        return self._head(x, None, fb, return_hidden, return_both, return_residual)

    # ------------------------------------------------------------------ dense forward
    @torch.no_grad()
    def forward_dense(self, tokens: torch.Tensor, cache, return_hidden: bool = False, bidirectional: bool = False):
        cfg = self.cfg
        Lq = tokens.shape[0]
        p0 = cache.offset
        positions = torch.arange(p0, p0 + Lq, dtype=torch.int32, device=tokens.device)
        x = ops.embedding(tokens.to(torch.int32), self.embed, cfg.embed_scale)
        ple = self._ple_inputs(tokens, x) if self.ple_dim else None
        for li, L in enumerate(self.layers):
            kvh, D, win = self.geom(li)
            H = self.H
            h = ops.rmsnorm(x, L.ln1, cfg.rms_norm_eps)
            packed = self._qkv_parts(L, li, h)
            cs, rd = self._rope(li)
            q, k, v = ops.qk_norm_rope_kv(packed, positions, None, cs, rd, False, L.q_norm, L.k_norm,
                                          cfg.rms_norm_eps, None, None, H, kvh, D, return_kv=True)
            ki = self.kv_index[li]
            if self.kv_owner[li]:
                kk, vv = cache.update(ki, k, v)
            else:
                kk, vv = cache.k[ki], cache.v[ki]
            a = ref.attention_rows_ref(q.float(), kk.float(), vv.float(), positions, kk.shape[0], cfg.scale,
                                       -1 if bidirectional else win, None, 0.0).to(x.dtype)
            x = self._block_tail(L, li, x, ops.gemm(a.reshape(Lq, H * D).contiguous(), L.wo), ple)
        cache.offset += Lq
        h = ops.rmsnorm(x, self.norm, cfg.rms_norm_eps)
        if return_hidden:
            return h
        return self._final_logits(h)

    def clone_to(self, device, dtype) -> "Gemma4LM":
        m = super().clone_to(device, dtype)
        for n in ("embed_ple", "ple_proj", "ple_proj_norm"):
            t = getattr(self, n)
            setattr(m, n, None if t is None else t.to(device=torch.device(device), dtype=dtype))
        return m


def build_from_tensors(cfg: DecoderConfig, ck, tensors: dict, device, dtype) -> Gemma4LM:
    """Gemma 4 weights from a checkpoint view (HF names, or MLX names with
    experts under ``switch_glu``). KV-shared layers' k/v projections and
    norms, when a checkpoint carries them, are not read
    (MLXLLM/Models/Gemma4Text.swift:2299-2345)."""
    from ..ops.qlinear import QuantizedWeight

    p = g4(cfg)
    m = Gemma4LM(cfg, "cpu", torch.float32)

    def vec(name):
        return ck.vec(name, required=True).float()

    def dense(w):
        return w.dequantize(torch.float32) if isinstance(w, QuantizedWeight) else w

    m.embed = ck.embedding("embed_tokens")
    m.norm = vec("norm.weight")
    m.lm_head = m.embed if (cfg.tie_word_embeddings or not ck.has("lm_head.weight")) else ck.linear("lm_head")
    if m.ple_dim:
        m.embed_ple = dense(ck.embedding("embed_tokens_per_layer"))
        m.ple_proj = ck.linear("per_layer_model_projection", packed=False)
        m.ple_proj_norm = vec("per_layer_projection_norm.weight")
    for li in range(cfg.num_layers):
        pre = f"layers.{li}."
        a = pre + "self_attn."
        L = LayerWeights()
        L.ln1 = vec(pre + "input_layernorm.weight")
        L.post_attn_norm = vec(pre + "post_attention_layernorm.weight")
        L.ln2 = vec(pre + "pre_feedforward_layernorm.weight")
        L.post_ffn_norm = vec(pre + "post_feedforward_layernorm.weight")
        parts = [ck.linear(a + "q_proj", packed=False)]
        if m.kv_owner[li]:
            parts.append(ck.linear(a + "k_proj", packed=False))
            if not (p["k_eq_v"] and m.kinds[li] == "full"):
                parts.append(ck.linear(a + "v_proj", packed=False))
            L.k_norm = vec(a + "k_norm.weight")
        L.wqkv = torch.cat([dense(t) for t in parts], 0)
        L.q_norm = vec(a + "q_norm.weight")
        L.wo = ck.linear(a + "o_proj", packed=False)
        mp = pre + "mlp."
        L.wgu = ref.interleave_gate_up(dense(ck.linear(mp + "gate_proj", packed=False)),
                                       dense(ck.linear(mp + "up_proj", packed=False)))
        L.wd = ck.linear(mp + "down_proj", packed=False)
        if p["moe"]:
            L.router = ck.linear(pre + "router.proj", packed=False)
            L.g4_router_scale = vec(pre + "router.scale")
            L.g4_expert_scale = vec(pre + "router.per_expert_scale")
            if ck.has(pre + "experts.gate_up_proj"):  # HF: [E, 2F, hidden] gate rows then up rows
                gu = ck.raw(pre + "experts.gate_up_proj").float()
                g, u = gu.chunk(2, 1)
                dn = ck.raw(pre + "experts.down_proj").float()
            else:  # MLX SwitchGLU stacks
                sg = pre + "experts.switch_glu."
                g = dense(ck.linear(sg + "gate_proj", packed=False))
                u = dense(ck.linear(sg + "up_proj", packed=False))
                dn = dense(ck.linear(sg + "down_proj", packed=False))
            L.experts_gu = torch.stack([ref.interleave_gate_up(g[e], u[e]) for e in range(g.shape[0])])
            L.experts_d = dn.contiguous()
            L.g4_post_ffn1 = vec(pre + "post_feedforward_layernorm_1.weight")
            L.g4_pre_ffn2 = vec(pre + "pre_feedforward_layernorm_2.weight")
            L.g4_post_ffn2 = vec(pre + "post_feedforward_layernorm_2.weight")
        if m.ple_dim:
            L.ple_gate = ck.linear(pre + "per_layer_input_gate", packed=False)
            L.ple_proj = ck.linear(pre + "per_layer_projection", packed=False)
            L.ple_norm = vec(pre + "post_per_layer_input_norm.weight")
        L.layer_scalar = ck.raw(pre + "layer_scalar").float().reshape(1) if ck.has(pre + "layer_scalar") \
            else torch.ones(1)
        m.layers.append(L)
    return m.clone_to(device, dtype)
