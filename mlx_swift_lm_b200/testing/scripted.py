"""Test support: a scripted language model and tokenizer (no weights).

Parity: Libraries/MLXScriptedLM (ScriptedTokenizer.swift:11, scripted models
whose output is fixed in advance) - engine, server and parser tests drive
the real scheduler, KV accounting, sampler, detokenizer and stream code with
a model whose next token is known.

:class:`ScriptedLM` is a :class:`DecoderLM` whose forward ignores its weights:
the logits of a row whose last token sits at position p put all mass on
``script[(p + 1 - prompt_len) % len(script)]`` (prompt_len is taken from the
first row it sees). Each call still writes nothing to the KV cache, so
paging, preemption and graph-free decoding run unchanged around it.
"""
from __future__ import annotations

import torch

from ..api.tokenizer import ByteTokenizer
from ..models.config import DecoderConfig
from ..models.decoder import DecoderLM


def scripted_tokenizer(vocab_size: int = 512) -> ByteTokenizer:
    return ByteTokenizer(vocab_size)


class ScriptedLM(DecoderLM):
    def __init__(self, script: list[int], prompt_len: int, vocab_size: int = 512, device="cpu"):
        cfg = DecoderConfig(model_type="scripted", vocab_size=vocab_size, hidden_size=64, num_layers=1, num_heads=1,
                            num_kv_heads=1, head_dim=64, intermediate_size=128, max_position_embeddings=1 << 16)
        super().__init__(cfg, device, torch.float32)
        self.init_random(0)
        self.script = list(script)
        self.prompt_len = prompt_len

    @classmethod
    def from_text(cls, text: str, prompt_len: int, tokenizer: ByteTokenizer | None = None):
        tok = tokenizer or scripted_tokenizer()
        return cls(tok.encode(text) + [tok.eos_token_id], prompt_len, tok.vocab_size)

    def _logits(self, positions: torch.Tensor) -> torch.Tensor:
        V = self.cfg.vocab_size
        idx = [(int(p) + 1 - self.prompt_len) % len(self.script) for p in positions.tolist()]
        out = torch.full((len(idx), V), -30.0, device=positions.device)
        out[torch.arange(len(idx)), torch.tensor([self.script[i] for i in idx])] = 30.0
        return out

    def forward(self, fb, kv, return_hidden=False, inputs_embeds=None, return_both=False, return_residual=False):
        pos = fb.positions if fb.logit_idx is None else fb.positions[fb.logit_idx]
        lg = self._logits(pos)
        h = torch.zeros(lg.shape[0], self.cfg.hidden_size, device=lg.device)
        if return_hidden:
            return h
        return (lg, h) if return_both else lg

    def forward_dense(self, tokens, cache, return_hidden=False):
        p0 = cache.offset
        cache.offset += tokens.shape[0]
        pos = torch.arange(p0, p0 + tokens.shape[0], device=tokens.device)
        return torch.zeros(len(pos), self.cfg.hidden_size) if return_hidden else self._logits(pos)
