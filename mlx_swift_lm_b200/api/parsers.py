"""Streaming reasoning and tool-call parsers.

Reasoning parsers split generated text into ``reasoning`` and ``content``:
  * ``think`` (deepseek_r1, qwen3): ``<think> ... </think>`` (the opening tag
    may be part of the prompt template, so text before ``</think>`` counts as
    reasoning when ``start_in_reasoning``);
  * ``harmony`` (gpt_oss): ``<|channel|>analysis<|message|> ... <|end|>``
    then ``<|channel|>final<|message|> ...``;
  * ``gemma4``: ``<start_of_thought> ... <end_of_thought>``.
Parity: MLXLMServer/Parsing/*ReasoningParser.swift, MLXLMCommon/ReasoningConfig.swift.

Tool-call parsers (one per model family's call syntax) live in
:mod:`.tool_formats`; ``make_tool_parser(name, tools)`` picks one.
Parity: MLXLMCommon/Tool/ToolCallFormat.swift:106-185, ToolCallProcessor.swift.
Parsers work incrementally: ``feed(text)`` returns the deltas that are safe
to emit, holding back any suffix that could still start a tag.
"""
from __future__ import annotations



def _holdback(buf: str, tags) -> int:
    """Length of the longest suffix of buf that is a proper prefix of a tag."""
    best = 0
    for t in tags:
        for k in range(min(len(t) - 1, len(buf)), 0, -1):
            if buf.endswith(t[:k]):
                best = max(best, k)
                break
    return best


class ThinkReasoningParser:
    def __init__(self, start="<think>", end="</think>", start_in_reasoning: bool = False):
        self.start, self.end = start, end
        self.in_reasoning = start_in_reasoning
        self.buf = ""

    def feed(self, text: str) -> tuple[str, str]:
        """Returns (reasoning_delta, content_delta)."""
        self.buf += text
        r_out, c_out = [], []
        while True:
            if self.in_reasoning:
                i = self.buf.find(self.end)
                if i >= 0:
                    r_out.append(self.buf[:i])
                    self.buf = self.buf[i + len(self.end):]
                    self.in_reasoning = False
                    continue
                h = _holdback(self.buf, [self.end])
                r_out.append(self.buf[: len(self.buf) - h])
                self.buf = self.buf[len(self.buf) - h:]
                break
            i = self.buf.find(self.start)
            if i >= 0:
                c_out.append(self.buf[:i])
                self.buf = self.buf[i + len(self.start):]
                self.in_reasoning = True
                continue
            h = _holdback(self.buf, [self.start])
            c_out.append(self.buf[: len(self.buf) - h])
            self.buf = self.buf[len(self.buf) - h:]
            break
        return "".join(r_out), "".join(c_out)

    def flush(self) -> tuple[str, str]:
        b, self.buf = self.buf, ""
        return (b, "") if self.in_reasoning else ("", b)


class HarmonyReasoningParser:
    """GPT-OSS harmony channels: analysis -> reasoning, final -> content."""

    TAGS = ["<|channel|>", "<|message|>", "<|end|>", "<|start|>", "<|return|>", "<|call|>"]

    def __init__(self):
        self.buf = ""
        self.channel = None
        self.in_header = False

    def feed(self, text: str) -> tuple[str, str]:
        self.buf += text
        r, c = [], []
        while True:
            if self.in_header:
                i = self.buf.find("<|message|>")
                if i < 0:
                    break
                header = self.buf[:i]
                self.channel = header.strip().split()[0] if header.strip() else "final"
                self.buf = self.buf[i + len("<|message|>"):]
                self.in_header = False
                continue
            j = min([k for k in (self.buf.find(t) for t in self.TAGS) if k >= 0], default=-1)
            if j < 0:
                h = _holdback(self.buf, self.TAGS)
                body, self.buf = self.buf[: len(self.buf) - h], self.buf[len(self.buf) - h:]
                (r if self.channel == "analysis" else c).append(body) if self.channel in ("analysis", "final", None) else None
                break
            body = self.buf[:j]
            if self.channel in ("analysis",):
                r.append(body)
            elif self.channel in ("final", None):
                c.append(body)
            rest = self.buf[j:]
            if rest.startswith("<|channel|>"):
                self.buf = rest[len("<|channel|>"):]
                self.in_header = True
            else:
                tag = next(t for t in self.TAGS if rest.startswith(t))
                self.buf = rest[len(tag):]
                if tag in ("<|end|>", "<|call|>", "<|return|>"):
                    self.channel = None if tag != "<|end|>" else self.channel
        return "".join(r), "".join(c)

    def flush(self):
        b, self.buf = self.buf, ""
        return (b, "") if self.channel == "analysis" else ("", b)


REASONING_PARSERS = {
    "deepseek_r1": lambda: ThinkReasoningParser(start_in_reasoning=True),
    "qwen3": lambda: ThinkReasoningParser(),
    "think": lambda: ThinkReasoningParser(),
    "harmony": HarmonyReasoningParser,
    "gpt_oss": HarmonyReasoningParser,
    "gemma4": lambda: ThinkReasoningParser("<start_of_thought>", "<end_of_thought>"),
}


def make_reasoning_parser(name: str | None):
    if not name:
        return None
    if name not in REASONING_PARSERS:
        raise ValueError(f"unknown reasoning parser {name!r}; choose from {sorted(REASONING_PARSERS)}")
    return REASONING_PARSERS[name]()


# ----------------------------------------------------------------------------- tools
from .tool_formats import (TOOL_FORMATS, HarmonyToolParser, JSONToolParser, Llama3ToolParser,  # noqa: E402,F401
                           MistralToolParser, ToolCall, infer_tool_format)

TOOL_PARSERS = TOOL_FORMATS


class TaggedJSONToolParser(JSONToolParser):
    """``<tool_call>{json}</tool_call>`` blocks (Hermes / Qwen), no bare-JSON recovery."""

    bare_recovery = False


class JSONObjectToolParser:
    """A reply that is a JSON object (or list) of calls, optionally after a
    prefix tag (Llama 3 ``<|python_tag|>``, Mistral ``[TOOL_CALLS]``)."""

    def __init__(self, prefix: str = ""):
        self.inner = MistralToolParser() if prefix == "[TOOL_CALLS]" else Llama3ToolParser()

    def feed(self, text):
        return self.inner.feed(text)

    def flush(self):
        return self.inner.flush()

    def parse(self, text):
        return self.inner.parse(text)


def make_tool_parser(name: str | None, tools: list | None = None):
    if not name:
        return None
    if name not in TOOL_PARSERS:
        raise ValueError(f"unknown tool-call parser {name!r}; choose from {sorted(TOOL_PARSERS)}")
    return TOOL_PARSERS[name](tools)


def validate_tool_arguments(call: ToolCall, tools: list[dict] | None) -> list[str]:
    """Minimal JSON-schema check of a call against the declared tools
    (ToolSchemaValidator.swift:20): known name, required keys, primitive types."""
    if not tools:
        return []
    spec = next((t.get("function", t) for t in tools if t.get("function", t).get("name") == call.name), None)
    if spec is None:
        return [f"unknown tool {call.name!r}"]
    params = spec.get("parameters") or {}
    errs = []
    for r in params.get("required", []):
        if r not in call.arguments:
            errs.append(f"missing required argument {r!r}")
    types = {"string": str, "integer": int, "number": (int, float), "boolean": bool, "array": list, "object": dict}
    for k, v in call.arguments.items():
        t = (params.get("properties", {}).get(k) or {}).get("type")
        if t in types and not isinstance(v, types[t]):
            errs.append(f"argument {k!r} should be {t}")
    return errs
