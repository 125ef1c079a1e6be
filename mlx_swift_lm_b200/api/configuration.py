"""Model configuration, download and tokenizer-loading protocols.

Parity: MLXLMCommon/ModelConfiguration.swift:16 (an id + revision or a local
directory, a tokenizer source, default prompt, extra EOS tokens, stop
strings, EOS ids, tool-call format), ``ResolvedModelConfiguration`` and the
pluggable ``Downloader`` / ``TokenizerLoader`` protocols
(MLXLMCommon/Downloader.swift:16, TokenizerLoader.swift:4).

This machine has no network, and neither has a B200 serving box by
assumption: :class:`LocalDownloader` resolves ids against local roots and the
Hugging Face cache layout (``models--{org}--{name}/snapshots/{revision}``)
and never fetches. A deployment plugs its own :class:`Downloader` in.
"""
from __future__ import annotations

import fnmatch
import os
from dataclasses import dataclass, field
from typing import Callable, Protocol


class Downloader(Protocol):
    def download(self, id: str, revision: str | None = None, matching: list[str] | None = None,
                 use_latest: bool = False, progress: Callable[[float], None] | None = None) -> str:
        """Local directory holding the files of `id` at `revision`."""
        ...


class TokenizerLoader(Protocol):
    def load(self, directory: str):
        """A tokenizer (the :mod:`.tokenizer` adapters' interface)."""
        ...


class ModelNotFound(FileNotFoundError):
    pass


class LocalDownloader:
    """Resolve model ids on local disk only: ``<root>/<org>/<name>``,
    ``<root>/<name>`` and the HF hub cache under each root (default roots:
    $HF_HUB_CACHE, $HF_HOME/hub, ~/.cache/huggingface/hub)."""

    def __init__(self, roots: list[str] | None = None):
        if roots is None:
            roots = [os.environ.get("HF_HUB_CACHE", ""), os.path.join(os.environ.get("HF_HOME", ""), "hub"),
                     os.path.expanduser("~/.cache/huggingface/hub")]
        self.roots = [r for r in roots if r]

    def download(self, id: str, revision: str | None = None, matching: list[str] | None = None,
                 use_latest: bool = False, progress=None) -> str:
        rev = revision or "main"
        for root in self.roots:
            for cand in (os.path.join(root, id), os.path.join(root, id.split("/")[-1])):
                if os.path.isdir(cand) and _has(cand, matching):
                    if progress:
                        progress(1.0)
                    return cand
            hub = os.path.join(root, "models--" + id.replace("/", "--"))
            if os.path.isdir(hub):
                ref = os.path.join(hub, "refs", rev)
                snap = open(ref).read().strip() if os.path.exists(ref) else rev
                d = os.path.join(hub, "snapshots", snap)
                if os.path.isdir(d) and _has(d, matching):
                    if progress:
                        progress(1.0)
                    return d
        raise ModelNotFound(f"{id}@{rev} is not on local disk (searched {self.roots}); this build never downloads")


def _has(d: str, matching: list[str] | None) -> bool:
    if not matching:
        return True
    names = os.listdir(d)
    return all(any(fnmatch.fnmatch(n, p) for n in names) for p in matching)


class HFTokenizerLoader:
    """A local ``transformers`` tokenizer (no network); falls back to the
    byte-level tokenizer when the directory has none."""

    def load(self, directory: str):
        from ..loader.load import load_tokenizer
        from .tokenizer import ByteTokenizer, as_tokenizer

        tok = load_tokenizer(directory)
        return as_tokenizer(tok) if tok is not None else ByteTokenizer()


@dataclass
class ResolvedModelConfiguration:
    model_directory: str
    tokenizer_directory: str
    name: str
    default_prompt: str = ""
    extra_eos_tokens: set = field(default_factory=set)
    stop_strings: set = field(default_factory=set)
    eos_token_ids: set = field(default_factory=set)
    tool_call_format: str | None = None
    reasoning_parser: str | None = None


@dataclass
class ModelConfiguration:
    """A model by hub id (+ revision) or by local directory."""
    id: str | None = None
    revision: str = "main"
    directory: str | None = None
    tokenizer_source: str | None = None  # id or directory of a separate tokenizer
    default_prompt: str = "hello"
    extra_eos_tokens: set = field(default_factory=set)
    stop_strings: set | None = None
    eos_token_ids: set = field(default_factory=set)
    tool_call_format: str | None = None
    reasoning_parser: str | None = None

    @property
    def name(self) -> str:
        if self.id:
            return self.id
        d = os.path.normpath(self.directory or "")
        return os.path.join(os.path.basename(os.path.dirname(d)), os.path.basename(d))

    @property
    def effective_stop_strings(self) -> set:
        return self.stop_strings if self.stop_strings is not None else set(self.extra_eos_tokens)

    def resolve(self, downloader: Downloader | None = None) -> ResolvedModelConfiguration:
        dl = downloader or LocalDownloader()
        model_dir = self.directory or dl.download(self.id, self.revision, ["config.json"])
        tok_dir = model_dir
        if self.tokenizer_source:
            tok_dir = (self.tokenizer_source if os.path.isdir(self.tokenizer_source)
                       else dl.download(self.tokenizer_source, None))
        return ResolvedModelConfiguration(model_dir, tok_dir, self.name, self.default_prompt,
                                          set(self.extra_eos_tokens), set(self.effective_stop_strings),
                                          set(self.eos_token_ids), self.tool_call_format, self.reasoning_parser)


# Known configurations (the reference's LLMRegistry entries for the families
# this framework benchmarks); any other id works through ModelConfiguration.
REGISTRY: dict[str, ModelConfiguration] = {
    c.id: c for c in (
        ModelConfiguration("Qwen/Qwen3-8B", tool_call_format="hermes", reasoning_parser="think"),
        ModelConfiguration("Qwen/Qwen3-30B-A3B", tool_call_format="hermes", reasoning_parser="think"),
        ModelConfiguration("Qwen/Qwen3-Next-80B-A3B-Instruct", tool_call_format="hermes"),
        ModelConfiguration("openai/gpt-oss-120b", tool_call_format="harmony", reasoning_parser="harmony",
                           extra_eos_tokens={"<|call|>", "<|return|>"}),
        ModelConfiguration("meta-llama/Meta-Llama-3-70B-Instruct", extra_eos_tokens={"<|eot_id|>"}),
        ModelConfiguration("mlx-community/Qwen3-4B-4bit", tool_call_format="hermes", reasoning_parser="think"),
    )
}


def configuration(id_or_dir: str) -> ModelConfiguration:
    """A registered configuration, a local directory, or a bare hub id."""
    if id_or_dir in REGISTRY:
        return REGISTRY[id_or_dir]
    if os.path.isdir(id_or_dir):
        return ModelConfiguration(directory=id_or_dir)
    return ModelConfiguration(id=id_or_dir)
