"""Tokenizer adapters.

* :class:`HFTokenizer` wraps a local ``transformers`` tokenizer (no network),
  including its chat template.
* :class:`ByteTokenizer` is a dependency-free byte-level tokenizer with a
  ChatML template, used by tests and synthetic models (the role of the
  reference's scripted tokenizer, Libraries/MLXScriptedLM/ScriptedTokenizer.swift:11).
"""
from __future__ import annotations

import json


class ByteTokenizer:
    """ids 0..255 are bytes; specials follow."""

    SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>", "<tool_call>", "</tool_call>"]
    # markup tokens stay in decoded text even with skip_special_tokens (as in
    # the Qwen tokenizers, where they are added but not special tokens)
    KEPT = {"<think>", "</think>", "<tool_call>", "</tool_call>"}

    def __init__(self, vocab_size: int = 512):
        self.vocab_size = max(vocab_size, 256 + len(self.SPECIALS))
        self.special_ids = {s: 256 + i for i, s in enumerate(self.SPECIALS)}
        self.id_to_special = {v: k for k, v in self.special_ids.items()}
        self.eos_token_id = self.special_ids["<|im_end|>"]
        self.bos_token_id = None
        self.pad_token_id = self.special_ids["<|endoftext|>"]

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        out = []
        i = 0
        while i < len(text):
            for s, sid in self.special_ids.items():
                if text.startswith(s, i):
                    out.append(sid)
                    i += len(s)
                    break
            else:
                out.extend(text[i].encode("utf-8"))
                i += 1
        return out

    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        buf = bytearray()
        parts = []
        for t in ids:
            t = int(t)
            if t < 256:
                buf.append(t)
            else:
                parts.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
                sp = self.id_to_special.get(t)
                if sp is not None and (not skip_special_tokens or sp in self.KEPT):
                    parts.append(sp)
        parts.append(buf.decode("utf-8", errors="replace"))
        return "".join(parts)

    def convert_ids_to_tokens(self, i: int) -> str:
        return self.id_to_special.get(i) or bytes([i]).decode("latin-1") if i < 256 else self.id_to_special.get(i, "")

    def apply_chat_template(self, messages, tools=None, add_generation_prompt=True, tokenize=False, **kw):
        s = ""
        if tools:
            s += "<|im_start|>system\n# Tools\n" + json.dumps(tools) + "<|im_end|>\n"
        for m in messages:
            content = m.get("content") or ""
            if isinstance(content, list):
                content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
            s += f"<|im_start|>{m['role']}\n{content}<|im_end|>\n"
        if add_generation_prompt:
            s += "<|im_start|>assistant\n"
        return self.encode(s) if tokenize else s

    def get_vocab_strings(self) -> list[str]:
        return [self.decode([i]) if i < 256 else self.id_to_special.get(i, "") for i in range(self.vocab_size)]


class HFTokenizer:
    def __init__(self, tok):
        self.tok = tok
        self.eos_token_id = tok.eos_token_id
        self.bos_token_id = getattr(tok, "bos_token_id", None)
        self.vocab_size = len(tok)

    @classmethod
    def from_dir(cls, path: str):
        from transformers import AutoTokenizer

        return cls(AutoTokenizer.from_pretrained(path, local_files_only=True))

    def encode(self, text, add_special_tokens=False):
        return self.tok.encode(text, add_special_tokens=add_special_tokens)

    def decode(self, ids, skip_special_tokens=False):
        return self.tok.decode(list(ids), skip_special_tokens=skip_special_tokens)

    def apply_chat_template(self, messages, tools=None, add_generation_prompt=True, tokenize=False, **kw):
        return self.tok.apply_chat_template(messages, tools=tools, add_generation_prompt=add_generation_prompt,
                                            tokenize=tokenize, **kw)

    def get_vocab_strings(self) -> list[str]:
        inv = {v: k for k, v in self.tok.get_vocab().items()}
        out = []
        for i in range(self.vocab_size):
            piece = inv.get(i, "")
            try:
                out.append(self.tok.convert_tokens_to_string([piece]) if piece else "")
            except Exception:
                out.append(piece)
        return out


def as_tokenizer(tok):
    if tok is None or isinstance(tok, (ByteTokenizer, HFTokenizer)):
        return tok
    return HFTokenizer(tok)
