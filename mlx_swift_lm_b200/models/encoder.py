"""Bidirectional encoders for embeddings and reranking: BERT, RoBERTa /
XLM-RoBERTa, DistilBERT and NomicBERT.

Parity: MLXEmbedders/Models/Bert.swift and NomicBert.swift (the embedder
model zoo of MLXEmbedders/ModelFactory.swift:31-47) and the cross-encoder
heads of MLXEmbedders/Reranker.swift.

B200 path: the same kernels as the decoder. A batch of sequences is packed
into one [T, H] activation; q|k|v come from one fused GEMM (bias epilogue),
K/V are written into a scratch paged cache and attention is the tensor-core
paged prefill kernel in bidirectional mode (``window = -1``); the FFN GEMM
applies GELU (or the SwiGLU of NomicBERT) in its epilogue; residual + LayerNorm
is one fused kernel. CPU tensors take the fp32 oracles of the same ops.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops
from ..kv.paged import PAGE
from ..ops import reference as ref
from .rope import build_rope


@dataclass
class EncoderConfig:
    model_type: str = "bert"  # bert | roberta | xlm-roberta | distilbert | nomic_bert
    vocab_size: int = 30522
    hidden_size: int = 384
    num_layers: int = 6
    num_heads: int = 12
    intermediate_size: int = 1536
    max_position_embeddings: int = 512
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12
    hidden_act: str = "gelu"  # gelu | gelu_tanh | swiglu
    rotary: bool = False  # NomicBERT: rotary positions instead of a position table
    rope_theta: float = 10000.0
    position_offset: int = 0  # RoBERTa family: positions start at padding_idx + 1
    bias: bool = True  # projection / FFN biases
    num_labels: int = 0  # > 0: sequence-classification head (cross-encoder rerankers)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @classmethod
    def from_hf(cls, hf: dict) -> "EncoderConfig":
        mt = hf.get("model_type", "bert")
        c = cls(model_type=mt, vocab_size=hf["vocab_size"])
        if mt == "distilbert":
            c.hidden_size, c.num_layers, c.num_heads = hf["dim"], hf["n_layers"], hf["n_heads"]
            c.intermediate_size = hf["hidden_dim"]
            c.type_vocab_size = 0
            c.layer_norm_eps = 1e-12
            c.hidden_act = "gelu" if hf.get("activation", "gelu") == "gelu" else "gelu_tanh"
        elif mt == "nomic_bert":
            c.hidden_size, c.num_layers, c.num_heads = hf["n_embd"], hf["n_layer"], hf["n_head"]
            c.intermediate_size = hf.get("n_inner") or 4 * c.hidden_size
            c.layer_norm_eps = hf.get("layer_norm_epsilon", 1e-12)
            c.rotary, c.rope_theta = True, hf.get("rotary_emb_base", 1000.0)
            c.hidden_act = "swiglu"
            c.bias = bool(hf.get("qkv_proj_bias", False))
            c.type_vocab_size = hf.get("type_vocab_size", 2)
        else:
            c.hidden_size, c.num_layers = hf["hidden_size"], hf["num_hidden_layers"]
            c.num_heads, c.intermediate_size = hf["num_attention_heads"], hf["intermediate_size"]
            c.type_vocab_size = hf.get("type_vocab_size", 2)
            c.layer_norm_eps = hf.get("layer_norm_eps", 1e-12)
            act = hf.get("hidden_act", "gelu")
            c.hidden_act = "gelu" if act == "gelu" else "gelu_tanh"
            if mt in ("roberta", "xlm-roberta", "camembert"):
                c.position_offset = hf.get("pad_token_id", 1) + 1
        c.max_position_embeddings = hf.get("max_position_embeddings", hf.get("n_positions", 512))
        labels = hf.get("id2label")
        if hf.get("architectures") and any("SequenceClassification" in a for a in hf["architectures"]):
            c.num_labels = len(labels) if labels else hf.get("num_labels", 1)
        return c


def scratch_layout(lens: list[int], device):
    """Page table [R, max pages] and K/V slots [T] placing each of R
    sequences of `lens` tokens on its own consecutive scratch pages; returns
    (page_table, slots, cu, pages)."""
    npg = [(n + PAGE - 1) // PAGE for n in lens]
    pt = torch.zeros(len(lens), max(npg), dtype=torch.int32)
    T = sum(lens)
    slots = torch.empty(T, dtype=torch.int64)
    cu, p = [0], 0
    for r, n in enumerate(lens):
        pt[r, :npg[r]] = torch.arange(p, p + npg[r])
        slots[cu[-1]:cu[-1] + n] = torch.arange(n) + p * PAGE
        cu.append(cu[-1] + n)
        p += npg[r]
    return pt.to(device), slots.to(device), cu, p


class EncoderLayer:
    __slots__ = ("wqkv", "bqkv", "wo", "bo", "ln1_w", "ln1_b", "w1", "b1", "w2", "b2", "ln2_w", "ln2_b")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)


class EncoderModel:
    """Post-norm bidirectional transformer encoder over packed sequences."""

    def __init__(self, cfg: EncoderConfig, device="cpu", dtype=torch.float32):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.word = self.pos = self.type = None
        self.emb_ln_w = self.emb_ln_b = None
        self.layers: list[EncoderLayer] = []
        self.pooler_w = self.pooler_b = None  # BERT pooler (dense + tanh on [CLS])
        self.cls_dense_w = self.cls_dense_b = None  # RoBERTa classification head dense
        self.cls_w = self.cls_b = None  # classifier
        D = cfg.head_dim
        rot = D if cfg.rotary else 0
        if cfg.rotary:
            self.cos_sin, self.rot_dim = build_rope(D, cfg.rope_theta, None, cfg.max_position_embeddings, 1.0)
        else:
            self.cos_sin, self.rot_dim = torch.zeros(1, 2), rot
        self.cos_sin = self.cos_sin.to(self.device)

    # ------------------------------------------------------------------ weights
    def init_random(self, seed: int = 0, std: float = 0.02, num_labels: int | None = None):
        cfg = self.cfg
        g = torch.Generator(device=self.device).manual_seed(seed)
        dev, dt, H, F = self.device, self.dtype, cfg.hidden_size, cfg.intermediate_size

        def rn(*shape):
            return torch.empty(shape, device=dev, dtype=dt).normal_(0.0, std, generator=g)

        def ones(n):
            return torch.ones(n, device=dev, dtype=dt)

        self.word = rn(cfg.vocab_size, H)
        if not cfg.rotary:
            self.pos = rn(cfg.max_position_embeddings + cfg.position_offset, H)
        if cfg.type_vocab_size:
            self.type = rn(cfg.type_vocab_size, H)
        self.emb_ln_w, self.emb_ln_b = ones(H), rn(H)
        for _ in range(cfg.num_layers):
            L = EncoderLayer()
            L.wqkv = rn(3 * H, H)
            L.wo = rn(H, H)
            if cfg.hidden_act == "swiglu":
                L.w1 = ref.interleave_gate_up(rn(F, H), rn(F, H))
            else:
                L.w1 = rn(F, H)
            L.w2 = rn(H, F)
            if cfg.bias:
                L.bqkv, L.bo, L.b2 = rn(3 * H), rn(H), rn(H)
                L.b1 = rn(2 * F if cfg.hidden_act == "swiglu" else F)
            L.ln1_w, L.ln1_b, L.ln2_w, L.ln2_b = ones(H), rn(H), ones(H), rn(H)
            self.layers.append(L)
        n = num_labels if num_labels is not None else cfg.num_labels
        if n:
            cfg.num_labels = n
            self.pooler_w, self.pooler_b = rn(H, H), rn(H)
            self.cls_w, self.cls_b = rn(n, H), rn(n)
        return self

    def tensors(self):
        for n in ("word", "pos", "type", "emb_ln_w", "emb_ln_b", "pooler_w", "pooler_b", "cls_dense_w", "cls_dense_b",
                  "cls_w", "cls_b"):
            yield n, getattr(self, n)
        for i, L in enumerate(self.layers):
            for s in EncoderLayer.__slots__:
                yield f"layers.{i}.{s}", getattr(L, s)

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, input_ids: list[list[int]], token_type_ids: list[list[int]] | None = None):
        """Packed hidden states [T, H] of the sequences and their offsets cu [R+1]."""
        cfg = self.cfg
        dev = self.device
        lens = [len(s) for s in input_ids]
        R = len(lens)
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        T = cu[-1]
        ids = torch.tensor([t for s in input_ids for t in s], dtype=torch.int32, device=dev)
        pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens]).to(dev)
        x = ops.embedding(ids, self.word)
        if self.pos is not None:
            x = (x.float() + self.pos[(pos + cfg.position_offset).long()].float()).to(self.dtype)
        if self.type is not None:
            tt = (torch.tensor([t for s in token_type_ids for t in s], device=dev) if token_type_ids is not None
                  else torch.zeros(T, dtype=torch.long, device=dev))
            x = (x.float() + self.type[tt.long()].float()).to(self.dtype)
        x = ops.add_layernorm(x.contiguous(), None, self.emb_ln_w, self.emb_ln_b, cfg.layer_norm_eps)
        # scratch pages: each sequence on its own consecutive pages
        pt, slots, _, p = scratch_layout(lens, dev)
        NH, D = cfg.num_heads, cfg.head_dim
        kc = torch.zeros(p, NH, PAGE, D, dtype=self.dtype, device=dev)
        vc = torch.zeros_like(kc)
        cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
        pos0 = torch.zeros(R, dtype=torch.int32, device=dev)
        scale = 1.0 / math.sqrt(D)
        mlp_epi = {"gelu": "gelu", "gelu_tanh": "gelu_tanh", "swiglu": "swiglu"}[cfg.hidden_act]
        for L in self.layers:
            qkv = ops.gemm(x, L.wqkv, bias=L.bqkv)
            q = ops.qk_norm_rope_kv(qkv, pos, slots, self.cos_sin, self.rot_dim, False, None, None,
                                    cfg.layer_norm_eps, kc, vc, NH, NH, D)
            a = ops.paged_prefill(q, kc, vc, pt, cu_t, pos0, scale, -1, cu_q_host=cu)
            d = ops.gemm(a.reshape(T, NH * D), L.wo, bias=L.bo)
            x = ops.add_layernorm(x, d, L.ln1_w, L.ln1_b, cfg.layer_norm_eps, out=x)
            h = ops.gemm(x, L.w1, epi=mlp_epi, bias=L.b1)
            d = ops.gemm(h, L.w2, bias=L.b2)
            x = ops.add_layernorm(x, d, L.ln2_w, L.ln2_b, cfg.layer_norm_eps, out=x)
        return x, cu

    def classify(self, x: torch.Tensor, cu: list[int]) -> torch.Tensor:
        """Sequence-classification logits [R, num_labels] fp32 from the [CLS]
        rows: BERT (pooler dense + tanh, classifier) or RoBERTa (dense + tanh,
        out_proj)."""
        cls = x[torch.tensor(cu[:-1], device=x.device)].contiguous()
        if self.cls_dense_w is not None:
            h = torch.tanh(ops.gemm(cls, self.cls_dense_w, bias=self.cls_dense_b, epi="f32")).to(x.dtype)
        else:
            h = torch.tanh(ops.gemm(cls, self.pooler_w, bias=self.pooler_b, epi="f32")).to(x.dtype)
        # a handful of labels: [R, H] x [H, labels] in fp32 (below the GEMM
        # kernel's 8-row tile granularity; not a hot path)
        return h.float() @ self.cls_w.float().t() + self.cls_b.float()

    def pooled_output(self, x: torch.Tensor, cu: list[int]) -> torch.Tensor | None:
        if self.pooler_w is None:
            return None
        cls = x[torch.tensor(cu[:-1], device=x.device)].contiguous()
        return torch.tanh(ops.gemm(cls, self.pooler_w, bias=self.pooler_b, epi="f32")).to(x.dtype)

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_tensors(cls, cfg: EncoderConfig, t: dict, device="cpu", dtype=torch.float32) -> "EncoderModel":
        """HF checkpoint names of BERT / RoBERTa / XLM-R / DistilBERT /
        NomicBERT (with or without the architecture prefix)."""
        m = cls(cfg, "cpu", torch.float32)
        keys = list(t)
        pre = ""
        for cand in ("bert.", "roberta.", "distilbert.", "model.", ""):
            if any(k.startswith(cand + "embeddings.") or k.startswith(cand + "encoder.") or
                   k.startswith(cand + "transformer.") or k.startswith(cand + "emb_ln") for k in keys):
                pre = cand
                break

        def get(name, required=True):
            for k in (pre + name, name):
                if k in t:
                    return t[k].float()
            if required:
                raise KeyError(name)
            return None

        mt = cfg.model_type
        H, F = cfg.hidden_size, cfg.intermediate_size
        m.word = get("embeddings.word_embeddings.weight")
        m.pos = get("embeddings.position_embeddings.weight", required=not cfg.rotary)
        m.type = get("embeddings.token_type_embeddings.weight", required=False)
        if mt == "nomic_bert":
            m.emb_ln_w, m.emb_ln_b = get("emb_ln.weight"), get("emb_ln.bias", False)
        else:
            m.emb_ln_w, m.emb_ln_b = get("embeddings.LayerNorm.weight"), get("embeddings.LayerNorm.bias")
        for i in range(cfg.num_layers):
            L = EncoderLayer()
            if mt == "distilbert":
                p = f"transformer.layer.{i}."
                L.wqkv = torch.cat([get(p + f"attention.{n}_lin.weight") for n in ("q", "k", "v")])
                L.bqkv = torch.cat([get(p + f"attention.{n}_lin.bias") for n in ("q", "k", "v")])
                L.wo, L.bo = get(p + "attention.out_lin.weight"), get(p + "attention.out_lin.bias")
                L.ln1_w, L.ln1_b = get(p + "sa_layer_norm.weight"), get(p + "sa_layer_norm.bias")
                L.w1, L.b1 = get(p + "ffn.lin1.weight"), get(p + "ffn.lin1.bias")
                L.w2, L.b2 = get(p + "ffn.lin2.weight"), get(p + "ffn.lin2.bias")
                L.ln2_w, L.ln2_b = get(p + "output_layer_norm.weight"), get(p + "output_layer_norm.bias")
            elif mt == "nomic_bert":
                p = f"encoder.layers.{i}."
                L.wqkv, L.bqkv = get(p + "attn.Wqkv.weight"), get(p + "attn.Wqkv.bias", False)
                L.wo, L.bo = get(p + "attn.out_proj.weight"), get(p + "attn.out_proj.bias", False)
                L.ln1_w, L.ln1_b = get(p + "norm1.weight"), get(p + "norm1.bias", False)
                up, gate = get(p + "mlp.fc11.weight"), get(p + "mlp.fc12.weight")
                L.w1 = ref.interleave_gate_up(gate, up)
                L.w2, L.b2 = get(p + "mlp.fc2.weight"), get(p + "mlp.fc2.bias", False)
                L.ln2_w, L.ln2_b = get(p + "norm2.weight"), get(p + "norm2.bias", False)
            else:
                p = f"encoder.layer.{i}."
                a = p + "attention."
                L.wqkv = torch.cat([get(a + f"self.{n}.weight") for n in ("query", "key", "value")])
                L.bqkv = torch.cat([get(a + f"self.{n}.bias") for n in ("query", "key", "value")])
                L.wo, L.bo = get(a + "output.dense.weight"), get(a + "output.dense.bias")
                L.ln1_w, L.ln1_b = get(a + "output.LayerNorm.weight"), get(a + "output.LayerNorm.bias")
                L.w1, L.b1 = get(p + "intermediate.dense.weight"), get(p + "intermediate.dense.bias")
                L.w2, L.b2 = get(p + "output.dense.weight"), get(p + "output.dense.bias")
                L.ln2_w, L.ln2_b = get(p + "output.LayerNorm.weight"), get(p + "output.LayerNorm.bias")
            m.layers.append(L)
        m.pooler_w, m.pooler_b = get("pooler.dense.weight", False), get("pooler.dense.bias", False)
        if "classifier.dense.weight" in t:  # RoBERTa / XLM-R classification head
            m.cls_dense_w, m.cls_dense_b = t["classifier.dense.weight"].float(), t["classifier.dense.bias"].float()
            m.cls_w, m.cls_b = t["classifier.out_proj.weight"].float(), t["classifier.out_proj.bias"].float()
        elif "classifier.weight" in t:
            m.cls_w, m.cls_b = t["classifier.weight"].float(), t["classifier.bias"].float()
        if m.cls_w is not None:
            cfg.num_labels = m.cls_w.shape[0]
        return m.to(device, dtype)

    def to(self, device, dtype):
        self.device, self.dtype = torch.device(device), dtype
        for n, v in list(self.tensors()):
            if v is None:
                continue
            if n.startswith("layers."):
                i, s = n.split(".")[1:]
                setattr(self.layers[int(i)], s, v.to(self.device, dtype).contiguous())
            else:
                setattr(self, n, v.to(self.device, dtype).contiguous())
        self.cos_sin = self.cos_sin.to(self.device)
        return self
