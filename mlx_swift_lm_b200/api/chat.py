"""ChatSession: multi-turn chat over a ModelContainer.

Parity: MLXLMCommon/ChatSession.swift:151-1736 - ``respond`` (:797),
``streamResponse`` (:871), ``streamDetails`` (:912), instructions, tools with
dispatch, ``saveCache`` (:1724), fork; the KV-reuse ledger (``cachedTokens``).

KV reuse across turns comes from the engine's prefix cache: each turn's
prompt is the whole conversation, so the previous turns' full blocks are
served from resident pages (``cached_tokens`` reports how many).
"""
from __future__ import annotations

import copy
import json

from ..engine.engine import EngineConfig
from .generate import GenerateParameters, generate_stream


class ChatSession:
    def __init__(self, container, instructions: str | None = None, params: GenerateParameters | None = None,
                 tools: list[dict] | None = None, tool_dispatch=None, tool_parser=None, reasoning_parser=None):
        self.container = container
        self.instructions = instructions
        self.params = params or GenerateParameters()
        self.tools = tools
        self.tool_dispatch = tool_dispatch  # callable(name, arguments: dict) -> str
        self.tool_parser = tool_parser
        self.reasoning_parser = reasoning_parser
        self.messages: list[dict] = []
        if instructions:
            self.messages.append({"role": "system", "content": instructions})
        self.cached_tokens = 0
        self.last_usage = None
        eng = container.engine
        if eng.prefix_cache is None:
            from ..kv.prefix_cache import PrefixCache

            eng.prefix_cache = PrefixCache(eng.kv, block_size=64)
            eng.sched.prefix_cache = eng.prefix_cache
            eng.sched.cfg.enable_prefix_cache = True

    def _run(self, stream_text: bool):
        toks = self.container.apply_chat_template(self.messages, tools=self.tools)
        out_toks, chunks, info = [], [], None
        for g in generate_stream(self.container.engine, toks, self.params):
            if g.token is not None:
                out_toks.append(g.token)
            if g.chunk:
                chunks.append(g.chunk)
                if stream_text:
                    yield g.chunk
            if g.info is not None:
                info = g.info
        text = "".join(chunks)
        self.last_usage = info
        yield ("__done__", text, out_toks)

    def stream_response(self, prompt: str, role: str = "user"):
        """Yield text chunks of the assistant's reply (tool calls are dispatched
        and answered automatically when a dispatcher is configured)."""
        self.messages.append({"role": role, "content": prompt})
        for _ in range(8):  # bounded tool-call rounds
            text = None
            for item in self._run(stream_text=True):
                if isinstance(item, tuple) and item[0] == "__done__":
                    text = item[1]
                else:
                    yield item
            calls = self.tool_parser.parse(text)[1] if (self.tool_parser and text) else []
            self.messages.append({"role": "assistant", "content": text,
                                  **({"tool_calls": [c.to_openai() for c in calls]} if calls else {})})
            if not calls or self.tool_dispatch is None:
                return
            for c in calls:
                result = self.tool_dispatch(c.name, c.arguments)
                self.messages.append({"role": "tool", "name": c.name,
                                      "content": result if isinstance(result, str) else json.dumps(result)})

    def respond(self, prompt: str, role: str = "user") -> str:
        return "".join(self.stream_response(prompt, role))

    def stream_details(self, prompt: str):
        """Yield (kind, payload): ('chunk', text) ... then ('info', completion info)."""
        for c in self.stream_response(prompt):
            yield ("chunk", c)
        yield ("info", self.last_usage)

    def fork(self) -> "ChatSession":
        s = ChatSession(self.container, None, copy.deepcopy(self.params), self.tools, self.tool_dispatch,
                        self.tool_parser, self.reasoning_parser)
        s.messages = copy.deepcopy(self.messages)
        return s

    def clear(self):
        self.messages = [m for m in self.messages if m["role"] == "system"]

    def save(self, path: str):
        """Persist the transcript (KV pages stay resident in the prefix cache)."""
        with open(path, "w") as f:
            json.dump({"instructions": self.instructions, "messages": self.messages}, f)

    @classmethod
    def load(cls, container, path: str, **kw) -> "ChatSession":
        with open(path) as f:
            d = json.load(f)
        s = cls(container, d.get("instructions"), **kw)
        s.messages = d["messages"]
        return s


_ = EngineConfig
