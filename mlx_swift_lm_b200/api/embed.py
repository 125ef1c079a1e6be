"""Embedding and reranking API.

Parity: MLXEmbedders (EmbedderModelContainer.swift:29, Pooling.swift:12 -
strategies mean / cls / first / last / max / none, optional LayerNorm,
truncation to `dimension`, L2 normalisation; sentence-transformers
``1_Pooling/config.json``) and the rerankers (MLXEmbedders/Reranker.swift:
single-logit, class-logit, binary-margin and softmax-probability scores, with
an identity or sigmoid transform; MLXRerankers for decoder rerankers).

Two model kinds serve both:

* encoders (:class:`..models.encoder.EncoderModel`: BERT, RoBERTa / XLM-R,
  DistilBERT, NomicBERT) - bidirectional attention, pooled token states;
  cross-encoder rerankers through their classification head;
* decoders (:class:`..models.decoder.DecoderLM`, e.g. Qwen3-Embedding /
  Qwen3-Reranker) - one prefill pass per batch through the paged kernels,
  last-token pooling; a decoder reranker scores the "yes" vs "no" logits of
  the last position.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import numpy as np
import torch

STRATEGIES = ("mean", "cls", "first", "last", "max", "none")


@dataclass
class Pooling:
    strategy: str = "mean"
    dimension: int | None = None

    @classmethod
    def from_sentence_transformers(cls, cfg: dict) -> "Pooling":
        """Priority CLS > mean > max > last, else first (Pooling.swift:123)."""
        dim = cfg.get("word_embedding_dimension")
        for key, st in (("pooling_mode_cls_token", "cls"), ("pooling_mode_mean_tokens", "mean"),
                        ("pooling_mode_max_tokens", "max"), ("pooling_mode_lasttoken", "last")):
            if cfg.get(key):
                return cls(st, dim)
        return cls("first", dim)

    def __call__(self, x: torch.Tensor, cu: list[int], pooled: torch.Tensor | None = None,
                 normalize: bool = False, layer_norm: bool = False) -> torch.Tensor:
        """Pooled [R, H] fp32 from packed token states x [T, H] with row
        offsets cu."""
        R = len(cu) - 1
        xf = x.float()
        if self.strategy == "mean":
            out = torch.stack([xf[cu[r]:cu[r + 1]].mean(0) for r in range(R)])
        elif self.strategy == "max":
            out = torch.stack([xf[cu[r]:cu[r + 1]].amax(0) for r in range(R)])
        elif self.strategy == "last":
            out = xf[torch.tensor([c - 1 for c in cu[1:]], device=x.device)]
        elif self.strategy == "cls" and pooled is not None:
            out = pooled.float()
        elif self.strategy in ("first", "cls"):
            out = xf[torch.tensor(cu[:-1], device=x.device)]
        else:  # none
            out = pooled.float() if pooled is not None else xf
        if layer_norm:
            out = torch.nn.functional.layer_norm(out, (out.shape[-1],), eps=1e-5)
        if self.dimension:
            out = out[:, :self.dimension]
        if normalize:
            out = torch.nn.functional.normalize(out, dim=-1)
        return out


def decoder_last_hidden(model, seqs: list[list[int]]) -> torch.Tensor:
    """Final-normed hidden state of each sequence's last token [R, H], one
    prefill forward of a decoder over a scratch paged cache."""
    from ..kv.paged import PagedKVCache, SequenceKV
    from ..models.batch import ForwardBatch

    dev = model.device
    total = sum(len(s) for s in seqs)
    kv = PagedKVCache.for_model(model, max_tokens=total + 16 * len(seqs), max_seqs=len(seqs))
    ids, pos, slots, cu, p0 = [], [], [], [0], []
    kvs = []
    for s in seqs:
        sq = SequenceKV(kv)
        assert sq.ensure(len(s))
        kvs.append(sq)
        ids.extend(s)
        pos.extend(range(len(s)))
        slots.extend(sq.slots(0, len(s)))
        cu.append(cu[-1] + len(s))
        p0.append(0)
    maxp = max(len(sq.pages) for sq in kvs)
    pt = np.zeros((len(seqs), maxp), np.int32)
    for i, sq in enumerate(kvs):
        pt[i, :len(sq.pages)] = sq.pages
    i32 = dict(dtype=torch.int32, device=dev)
    fb = ForwardBatch(input_ids=torch.tensor(ids, **i32), positions=torch.tensor(pos, **i32),
                      slots=torch.tensor(slots, dtype=torch.int64, device=dev), num_decode=0)
    fb.pf_cu_q, fb.pf_cu_q_host = torch.tensor(cu, **i32), cu
    fb.pf_pos0 = torch.tensor(p0, **i32)
    fb.pf_page_table = torch.from_numpy(pt).to(dev)
    fb.logit_idx_host = [c - 1 for c in cu[1:]]
    fb.logit_idx = torch.tensor(fb.logit_idx_host, dtype=torch.int64, device=dev)
    if kv.rec is not None:
        fb.state_slots = torch.tensor([sq.state_slot for sq in kvs], **i32)
    with torch.no_grad():
        h = model.forward(fb, kv, return_hidden=True)
    for sq in kvs:
        sq.release()
    return h


class Embedder:
    """Sentence embeddings from an encoder or a decoder."""

    def __init__(self, model, pooling: Pooling | None = None, tokenizer=None, normalize: bool = True,
                 max_length: int | None = None):
        from ..models.encoder import EncoderModel

        self.model = model
        self.is_encoder = isinstance(model, EncoderModel)
        self.pooling = pooling or Pooling("mean" if self.is_encoder else "last")
        self.tokenizer = tokenizer
        self.normalize = normalize
        self.max_length = max_length or (model.cfg.max_position_embeddings if self.is_encoder else None)

    def _ids(self, inputs) -> list[list[int]]:
        out = []
        for x in inputs:
            if isinstance(x, str):
                if self.tokenizer is None:
                    raise ValueError("text input needs a tokenizer")
                x = self.tokenizer.encode(x, add_special_tokens=True) if self.is_encoder else self.tokenizer.encode(x)
            x = list(x)
            if self.max_length:
                x = x[:self.max_length]
            out.append(x)
        return out

    @torch.no_grad()
    def embed(self, inputs, normalize: bool | None = None, batch_size: int = 64) -> torch.Tensor:
        """Embeddings [N, dim] (fp32, on the model's device)."""
        ids = self._ids(inputs)
        norm = self.normalize if normalize is None else normalize
        outs = []
        for i in range(0, len(ids), batch_size):
            chunk = ids[i:i + batch_size]
            if self.is_encoder:
                x, cu = self.model.forward(chunk)
                outs.append(self.pooling(x, cu, self.model.pooled_output(x, cu), normalize=norm))
            else:
                h = decoder_last_hidden(self.model, chunk)
                cu = list(range(h.shape[0] + 1))
                outs.append(Pooling("first", self.pooling.dimension)(h, cu, normalize=norm))
        return torch.cat(outs, 0)

    @classmethod
    def from_pretrained(cls, path: str, device=None, dtype=torch.bfloat16, normalize: bool = True):
        """A local model directory: encoders by ``model_type`` (bert,
        roberta, xlm-roberta, distilbert, nomic_bert), anything else through
        the decoder loader; pooling from ``1_Pooling/config.json`` when present."""
        from ..loader.load import load_tokenizer
        from ..loader.safetensors import load_safetensors
        from ..models.encoder import EncoderConfig, EncoderModel

        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        if torch.device(device).type == "cpu":
            dtype = torch.float32
        hf = json.load(open(os.path.join(path, "config.json")))
        pooling = None
        pc = os.path.join(path, "1_Pooling", "config.json")
        if os.path.exists(pc):
            pooling = Pooling.from_sentence_transformers(json.load(open(pc)))
        if hf.get("model_type") in ENCODER_TYPES:
            cfg = EncoderConfig.from_hf(hf)
            model = EncoderModel.from_tensors(cfg, load_safetensors(path), device, dtype)
        else:
            from ..loader.load import load_model

            model, _ = load_model(path, device, dtype)
        try:
            tok = load_tokenizer(path)
        except Exception:
            tok = None
        return cls(model, pooling, tok, normalize)


ENCODER_TYPES = ("bert", "roberta", "xlm-roberta", "camembert", "distilbert", "nomic_bert")


@dataclass
class RerankScore:
    """How a reranker turns logits into a score (Reranker.swift:8-30):
    kind single_logit | class_logit | binary_margin | softmax_probability,
    transform identity | sigmoid."""
    kind: str = "single_logit"
    index: int = 0
    positive: int = 1
    negative: int = 0
    transform: str = "sigmoid"

    def __call__(self, logits: torch.Tensor) -> list[float]:
        lg = logits.float()
        if self.kind == "single_logit":
            v = lg[:, 0]
        elif self.kind == "class_logit":
            v = lg[:, self.index]
        elif self.kind == "binary_margin":
            v = lg[:, self.positive] - lg[:, self.negative]
        else:  # softmax_probability
            return torch.softmax(lg, -1)[:, self.index].tolist()
        if self.transform == "sigmoid":
            v = torch.sigmoid(v)
        return v.tolist()


class Reranker:
    """Query-document relevance scores.

    Cross-encoder (encoder with a classification head): input
    ``[CLS] query [SEP] document [SEP]`` (token types 0 / 1), score from the
    head's logits. Decoder reranker (Qwen3-Reranker style): the prompt built
    by `template` and the softmax over the ("no", "yes") logits at the last
    position."""

    def __init__(self, model, tokenizer=None, score: RerankScore | None = None, yes_no: tuple[int, int] | None = None,
                 template=None, cls_id: int = 101, sep_id: int = 102):
        from ..models.encoder import EncoderModel

        self.model = model
        self.tokenizer = tokenizer
        self.is_encoder = isinstance(model, EncoderModel)
        self.score_fn = score or (RerankScore() if self.is_encoder else
                                  RerankScore("softmax_probability", index=1))
        self.yes_no = yes_no
        self.template = template
        self.cls_id, self.sep_id = cls_id, sep_id

    def _tok(self, t):
        if isinstance(t, str):
            if self.tokenizer is None:
                raise ValueError("text input needs a tokenizer")
            return list(self.tokenizer.encode(t))
        return list(t)

    @torch.no_grad()
    def score(self, query, documents: list) -> list[float]:
        q = self._tok(query)
        if self.is_encoder:
            ids, tts = [], []
            for d in documents:
                dd = self._tok(d)
                ids.append([self.cls_id] + q + [self.sep_id] + dd + [self.sep_id])
                tts.append([0] * (len(q) + 2) + [1] * (len(dd) + 1))
            x, cu = self.model.forward(ids, tts if self.model.type is not None else None)
            return self.score_fn(self.model.classify(x, cu))
        assert self.yes_no is not None, "a decoder reranker needs the (no, yes) token ids"
        seqs = [self.template(q, self._tok(d)) if self.template else q + self._tok(d) for d in documents]
        h = decoder_last_hidden(self.model, seqs)
        logits = self.model._final_logits(h)
        no, yes = self.yes_no
        return self.score_fn(logits[:, [no, yes]])
