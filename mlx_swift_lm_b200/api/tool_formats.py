"""Tool-call formats: one streaming parser per model family's call syntax.

Every parser takes generated text incrementally: ``feed(text)`` returns
``(content_delta, calls)`` - the text outside call frames that is safe to
emit now (a suffix that could still open a frame is held back) and the calls
whose frames closed in this piece - and ``flush()`` ends the stream (a frame
cut off by end-of-sequence is parsed as if closed). ``parse(text)`` runs a
whole reply. Argument values are typed by the declared tool schemas when the
syntax carries raw text (XML / key-value dialects): a parameter declared only
as ``string`` keeps its raw text, anything else is read as JSON when it
parses.

Formats (names as the reference's ``ToolCallFormat``,
MLXLMCommon/Tool/ToolCallFormat.swift:106-185):

==============  ==================================================================
json / hermes   ``<tool_call>{"name": f, "arguments": {...}}</tool_call>``; a reply that
                is only a JSON call object is recovered at the end
xml_function    ``<tool_call><function=f><parameter=k>v</parameter></function></tool_call>``
nemotron        xml_function, the outer ``<tool_call>`` wrapper optional
qwen3_5         ``<tool_call>`` frame holding either the XML function or the JSON payload
mimo_v2         xml_function frame (raw string values)
glm4            ``<tool_call>f<arg_key>k</arg_key><arg_value>v</arg_value></tool_call>``,
                or a declared tool's ``f\\n{json}`` without markers
glm5 / flint    the glm4 key/value frame only (strict)
gemma / gemma4  ``<|tool_call>call:f{k:<|"|>str<|"|>,n:3}<tool_call|>`` (gemma also
                ``<start_function_call>...<end_function_call>`` and ``<escape>`` quotes)
kimi_k2         ``<|tool_call_begin|>functions.f:0<|tool_call_argument_begin|>{json}<|tool_call_end|>``
minimax_m2      ``<minimax:tool_call><invoke name="f"><parameter name="k">v</parameter>
                </invoke></minimax:tool_call>``
atem            ``<atem:function_calls><atem:invoke name="f"><atem:parameter name="k">v
                </atem:parameter></atem:invoke></atem:function_calls>``
mistral         ``[TOOL_CALLS]f[CALL_ID]id[ARGS]{json}`` (v11+) or ``[TOOL_CALLS][{...}]``
llama3          ``<|python_tag|>{"name": f, "parameters": {...}}`` or the bare object(s)
lfm2            ``<|tool_call_start|>[f(a='x', b=2), g()]<|tool_call_end|>`` (Python call syntax)
gpt_oss/harmony ``<|channel|>commentary to=functions.f<|message|>{json}<|call|>``
==============  ==================================================================
"""
from __future__ import annotations

import ast
import json
import re
import uuid
from dataclasses import dataclass, field


@dataclass
class ToolCall:
    name: str
    arguments: dict
    id: str = field(default_factory=lambda: "call_" + uuid.uuid4().hex[:24])

    def to_openai(self) -> dict:
        return {"id": self.id, "type": "function",
                "function": {"name": self.name, "arguments": json.dumps(self.arguments)}}


def _holdback(buf: str, tags) -> int:
    """Length of the longest suffix of buf that is a proper prefix of a tag."""
    best = 0
    for t in tags:
        for k in range(min(len(t) - 1, len(buf)), 0, -1):
            if buf.endswith(t[:k]):
                best = max(best, k)
                break
    return best


def _loads(s):
    try:
        return json.loads(s)
    except Exception:
        return None


def _tool_schema(tools, name):
    for t in tools or []:
        f = t.get("function", t)
        if f.get("name") == name:
            return f.get("parameters") or {}
    return None


def _declared_types(schema) -> set:
    if not isinstance(schema, dict):
        return set()
    t = schema.get("type")
    out = set([t] if isinstance(t, str) else (t or []))
    for k in ("anyOf", "oneOf"):
        for br in schema.get(k, []) or []:
            out |= _declared_types(br)
    return out


def typed_value(raw: str, schema) -> object:
    """Raw argument text -> value: declared-string-only parameters keep the
    text; otherwise JSON when it parses (in a union with string, only as one
    of the other types), else the text."""
    types = _declared_types(schema)
    if types == {"string"}:
        return raw
    v = _loads(raw.strip())
    if v is None and raw.strip() != "null":
        return raw
    if "string" in types and isinstance(v, str):
        return raw
    return v


def _param_schema(tools, name, key):
    s = _tool_schema(tools, name)
    return (s or {}).get("properties", {}).get(key) if s else None


def _strip_nl(v: str) -> str:
    """Templates put the value on its own line: drop one leading / trailing newline."""
    if v.startswith("\n"):
        v = v[1:]
    if v.endswith("\n"):
        v = v[:-1]
    return v


# ============================================================================ framing
class FramedToolParser:
    """Streams text outside call frames; each closed frame's body goes to
    :meth:`parse_body`. ``frames`` maps start tag -> end tag (None: the frame
    runs to end-of-sequence or until :meth:`complete` says it is whole)."""

    frames: dict = {}
    drop_tags: tuple = ()  # section markers removed from content

    def __init__(self, tools: list | None = None):
        self.tools = tools
        self.buf = ""
        self.open: str | None = None  # start tag of the frame being read
        self._stash = ""  # content seen by feed(), for end-of-reply recovery

    # -- per format
    def parse_body(self, body: str, start: str) -> list[ToolCall]:
        raise NotImplementedError

    def complete(self, body: str, start: str) -> int | None:
        """For frames without an end tag: length of a whole call at the head of
        `body`, or None while it is still incomplete."""
        return None

    def recover(self, content: str) -> tuple[str, list[ToolCall]]:
        """End-of-reply recovery of calls written without frames."""
        return content, []

    # -- streaming
    def feed(self, text: str) -> tuple[str, list[ToolCall]]:
        self.buf += text
        out, calls = [], []
        while True:
            if self.open is not None:
                end = self.frames[self.open]
                if end is None:
                    n = self.complete(self.buf, self.open)
                    if n is None:
                        break
                    calls += self.parse_body(self.buf[:n], self.open)
                    self.buf = self.buf[n:]
                else:
                    i = self.buf.find(end)
                    if i < 0:
                        break
                    calls += self.parse_body(self.buf[:i], self.open)
                    self.buf = self.buf[i + len(end):]
                self.open = None
                continue
            hits = [(self.buf.find(s), s) for s in self.frames]
            hits = [(i, s) for i, s in hits if i >= 0]
            if hits:
                i, s = min(hits, key=lambda x: (x[0], -len(x[1])))
                out.append(self.buf[:i])
                self.buf = self.buf[i + len(s):]
                self.open = s
                continue
            h = _holdback(self.buf, list(self.frames) + list(self.drop_tags))
            out.append(self.buf[:len(self.buf) - h])
            self.buf = self.buf[len(self.buf) - h:]
            break
        content = "".join(out)
        for t in self.drop_tags:
            content = content.replace(t, "")
        self._stash += content
        return content, calls

    def flush(self) -> tuple[str, list[ToolCall]]:
        calls = []
        rest = self.buf
        if self.open is not None:
            calls = self.parse_body(rest, self.open)
            rest = "" if calls else self.open + rest
        self.buf, self.open = "", None
        for t in self.drop_tags:
            rest = rest.replace(t, "")
        return rest, calls

    def parse(self, text: str) -> tuple[str, list[ToolCall]]:
        p = type(self)(self.tools)
        c, calls = p.feed(text)
        c2, calls2 = p.flush()
        content, calls = c + c2, calls + calls2
        if not calls:
            return self.recover(content)
        return content, calls


# ============================================================================ JSON dialects
def _json_calls(obj, name_keys=("name",), arg_keys=("arguments", "parameters")) -> list[ToolCall]:
    objs = obj if isinstance(obj, list) else [obj]
    out = []
    for o in objs:
        if not isinstance(o, dict):
            continue
        if "function" in o and isinstance(o["function"], dict):  # OpenAI-shaped
            o = o["function"]
        name = next((o[k] for k in name_keys if isinstance(o.get(k), str)), None)
        if name is None:
            continue
        args = next((o[k] for k in arg_keys if k in o), {})
        if isinstance(args, str):
            args = _loads(args) or {}
        out.append(ToolCall(name, args if isinstance(args, dict) else {}))
    return out


class JSONToolParser(FramedToolParser):
    frames = {"<tool_call>": "</tool_call>"}
    bare_recovery = True

    def parse_body(self, body, start):
        return _json_calls(_loads(body.strip()))

    def recover(self, content):
        if not self.bare_recovery:
            return content, []
        calls = _json_calls(_loads(content.strip())) if content.strip()[:1] in "{[" else []
        return ("" if calls else content), calls


class Llama3ToolParser(FramedToolParser):
    frames = {"<|python_tag|>": None}

    def complete(self, body, start):
        return None  # runs to end-of-sequence

    def parse_body(self, body, start):
        calls = []
        for part in (p for p in re.split(r";\s*(?=\{)", body.strip()) if p.strip()):
            calls += _json_calls(_loads(part))
        return calls

    def recover(self, content):
        t = content.strip()
        if not t.startswith(("{", "[")):
            return content, []
        calls = self.parse_body(t, "")
        return ("" if calls else content), calls


class MistralToolParser(FramedToolParser):
    """v11+: ``[TOOL_CALLS]name[CALL_ID]id[ARGS]{json}`` (one frame per call);
    earlier: ``[TOOL_CALLS][{"name":..,"arguments":..}, ...]``."""

    frames = {"[TOOL_CALLS]": None}

    def complete(self, body, start):
        s = body.lstrip()
        lead = len(body) - len(s)
        if s.startswith("["):
            try:
                _, n = json.JSONDecoder().raw_decode(s)
                return lead + n
            except ValueError:
                return None
        i = s.find("[ARGS]")
        if i < 0:
            return None
        j = i + len("[ARGS]")
        a = s[j:]
        a_lead = len(a) - len(a.lstrip())
        try:
            _, n = json.JSONDecoder().raw_decode(a.lstrip())
        except ValueError:
            return None
        return lead + j + a_lead + n

    def parse_body(self, body, start):
        s = body.strip()
        if s.startswith("["):
            return _json_calls(_loads(s))
        i = s.find("[ARGS]")
        if i < 0:
            return []
        name, cid = s[:i].strip(), None
        if "[CALL_ID]" in name:
            name, cid = (x.strip() for x in name.split("[CALL_ID]", 1))
        args = _loads(s[i + len("[ARGS]"):].strip())
        if not name or not isinstance(args, dict):
            return []
        c = ToolCall(name, args)
        if cid:
            c.id = cid
        return [c]


# ============================================================================ XML dialects
_FUNC_RE = re.compile(r"<function=([^>\n]+)>(.*?)</function>", re.S)
_PARAM_RE = re.compile(r"<parameter=([^>\n]+)>(.*?)</parameter>", re.S)


def _xml_function_calls(body: str, tools) -> list[ToolCall]:
    calls = []
    for m in _FUNC_RE.finditer(body + ("</function>" if "<function=" in body and "</function>" not in body else "")):
        name = m.group(1).strip()
        args = {}
        for p in _PARAM_RE.finditer(m.group(2)):
            k = p.group(1).strip()
            args[k] = typed_value(_strip_nl(p.group(2)), _param_schema(tools, name, k))
        calls.append(ToolCall(name, args))
    return calls


class XMLFunctionToolParser(FramedToolParser):
    frames = {"<tool_call>": "</tool_call>"}

    def parse_body(self, body, start):
        if start == "<function=":
            body = "<function=" + body + "</function>"
        return _xml_function_calls(body, self.tools)


class NemotronToolParser(XMLFunctionToolParser):
    frames = {"<tool_call>": "</tool_call>", "<function=": "</function>"}


class Qwen35ToolParser(FramedToolParser):
    """Qwen 3.5 is prompted for the XML function payload and sometimes
    writes the Hermes JSON one inside the same frame; the payload's first
    character decides (Tool/Parsers/Qwen35ToolCallParser.swift:5-36)."""

    frames = {"<tool_call>": "</tool_call>"}

    def parse_body(self, body, start):
        s = body.strip()
        if s.startswith("<function="):
            return _xml_function_calls(s, self.tools)
        if s.startswith(("{", "[")):
            return _json_calls(_loads(s))
        return []


class MiMoV2ToolParser(XMLFunctionToolParser):
    pass


_KV_RE = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", re.S)


class GLM4ToolParser(FramedToolParser):
    frames = {"<tool_call>": "</tool_call>"}
    markerless = True

    def parse_body(self, body, start):
        s = body.strip()
        i = s.find("<arg_key>")
        if i < 0:
            if not self.markerless:
                name = s
                return [ToolCall(name, {})] if name and "\n" not in name and "{" not in name else []
            name, _, rest = s.partition("\n")
            name = name.strip()
            args = _loads(rest.strip()) if rest.strip() else {}
            if name and isinstance(args, dict) and (self.tools is None or _tool_schema(self.tools, name) is not None):
                return [ToolCall(name, args)]
            return []
        name = s[:i].strip()
        if not name:
            return []
        args = {}
        for m in _KV_RE.finditer(s[i:]):
            k = m.group(1).strip()
            args[k] = typed_value(m.group(2).strip() if self.markerless else m.group(2),
                                  _param_schema(self.tools, name, k))
        return [ToolCall(name, args)]


class GLM5ToolParser(GLM4ToolParser):
    markerless = False


class FlintToolParser(GLM4ToolParser):
    markerless = False


class MiniMaxM2ToolParser(FramedToolParser):
    frames = {"<minimax:tool_call>": "</minimax:tool_call>"}
    invoke, param, pfx = "invoke", "parameter", ""

    def parse_body(self, body, start):
        inv = re.compile(rf"<{self.pfx}{self.invoke} name=(\"[^\"]*\"|'[^']*'|[^>\s]+)\s*>(.*?)</{self.pfx}{self.invoke}>",
                         re.S)
        par = re.compile(rf"<{self.pfx}{self.param} name=(\"[^\"]*\"|'[^']*'|[^>\s]+)\s*>(.*?)</{self.pfx}{self.param}>",
                         re.S)
        calls = []
        for m in inv.finditer(body):
            name = m.group(1).strip("\"'")
            args = {}
            for p in par.finditer(m.group(2)):
                k = p.group(1).strip("\"'")
                args[k] = typed_value(_strip_nl(p.group(2).strip(" \t")), _param_schema(self.tools, name, k))
            calls.append(ToolCall(name, args))
        return calls


class ATEMToolParser(MiniMaxM2ToolParser):
    frames = {"<atem:function_calls>": "</atem:function_calls>"}
    pfx = "atem:"


class KimiK2ToolParser(FramedToolParser):
    frames = {"<|tool_call_begin|>": "<|tool_call_end|>"}
    drop_tags = ("<|tool_calls_section_begin|>", "<|tool_calls_section_end|>")

    def parse_body(self, body, start):
        head, sep, args = body.partition("<|tool_call_argument_begin|>")
        if not sep:
            return []
        head = head.strip()
        name = head.rsplit(":", 1)[0] if ":" in head else head
        if name.startswith("functions."):
            name = name[len("functions."):]
        elif "." in name:
            name = name.split(".", 1)[1]
        a = _loads(args.strip())
        if not name or not isinstance(a, dict):
            return []
        c = ToolCall(name, a)
        c.id = head if head.startswith("functions.") else c.id
        return [c]


# ============================================================================ Gemma
class _GemmaValues:
    """Recursive-descent reader of Gemma's call argument syntax:
    ``{key:value,...}`` with bare keys, ``<|"|>``/``<escape>``-quoted strings,
    JSON numbers / true / false / null, nested objects and lists."""

    QUOTES = ('<|"|>', "<escape>")

    def __init__(self, s: str):
        self.s, self.i = s, 0

    def ws(self):
        while self.i < len(self.s) and self.s[self.i].isspace():
            self.i += 1

    def value(self):
        self.ws()
        s = self.s
        for q in self.QUOTES:
            if s.startswith(q, self.i):
                j = s.find(q, self.i + len(q))
                if j < 0:
                    raise ValueError("unterminated string")
                v = s[self.i + len(q):j]
                self.i = j + len(q)
                return v
        c = s[self.i:self.i + 1]
        if c == "{":
            return self.obj()
        if c == "[":
            self.i += 1
            out = []
            self.ws()
            if s.startswith("]", self.i):
                self.i += 1
                return out
            while True:
                out.append(self.value())
                self.ws()
                if s.startswith(",", self.i):
                    self.i += 1
                    continue
                if s.startswith("]", self.i):
                    self.i += 1
                    return out
                raise ValueError("bad list")
        if c == '"':
            v, n = json.JSONDecoder().raw_decode(s[self.i:])
            self.i += n
            return v
        m = re.compile(r"[^,}\]]+").match(s, self.i)
        if not m:
            raise ValueError("empty value")
        tok = m.group(0).strip()
        self.i = m.end()
        v = _loads(tok)
        return tok if v is None and tok != "null" else v

    def obj(self):
        s = self.s
        assert s[self.i] == "{"
        self.i += 1
        out = {}
        self.ws()
        if s.startswith("}", self.i):
            self.i += 1
            return out
        while True:
            self.ws()
            m = re.compile(r"[^:{}\s]+").match(s, self.i)
            if not m:
                raise ValueError("bad key")
            key = m.group(0).strip('"')
            self.i = m.end()
            self.ws()
            if not s.startswith(":", self.i):
                raise ValueError("missing ':'")
            self.i += 1
            out[key] = self.value()
            self.ws()
            if s.startswith(",", self.i):
                self.i += 1
                continue
            if s.startswith("}", self.i):
                self.i += 1
                return out
            raise ValueError("bad object")


def _gemma_calls(body: str) -> list[ToolCall]:
    calls = []
    s = body.strip()
    while s.startswith("call:"):
        j = s.find("{")
        if j < 0:
            break
        name = s[len("call:"):j].strip()
        r = _GemmaValues(s)
        r.i = j
        try:
            args = r.obj()
        except (ValueError, AssertionError):
            break
        calls.append(ToolCall(name, args))
        s = s[r.i:].lstrip().lstrip(",").lstrip()
    return calls


class GemmaToolParser(FramedToolParser):
    frames = {"<|tool_call>": "<tool_call|>", "<start_function_call>": "<end_function_call>"}

    def parse_body(self, body, start):
        return _gemma_calls(body)


class Gemma4ToolParser(GemmaToolParser):
    frames = {"<|tool_call>": "<tool_call|>"}


# ============================================================================ Python call syntax
class PythonicToolParser(FramedToolParser):
    """``[f(a='x', b=2), g()]`` read with Python's own parser (literal values only)."""

    frames = {"<|tool_call_start|>": "<|tool_call_end|>"}

    def parse_body(self, body, start):
        s = body.strip()
        try:
            tree = ast.parse(s, mode="eval").body
        except SyntaxError:
            return []
        nodes = tree.elts if isinstance(tree, (ast.List, ast.Tuple)) else [tree]
        calls = []
        for n in nodes:
            if not isinstance(n, ast.Call):
                continue
            f = n.func
            name = f.id if isinstance(f, ast.Name) else (ast.unparse(f) if isinstance(f, ast.Attribute) else None)
            if not name:
                continue
            args = {}
            try:
                for kw in n.keywords:
                    if kw.arg is not None:
                        args[kw.arg] = ast.literal_eval(kw.value)
            except ValueError:
                continue
            calls.append(ToolCall(name, args))
        return calls


# ============================================================================ Harmony
class HarmonyToolParser:
    """``<|channel|>commentary to=functions.NAME<|constrain|>json<|message|>{...}<|call|>``
    (and the recipient in the ``<|start|>assistant to=functions.NAME`` header)."""

    PAT = re.compile(r"to=functions\.([\w\-\.]+)[^<]*(?:<\|channel\|>[^<]*)?(?:<\|constrain\|>\w+)?<\|message\|>(.*?)"
                     r"<\|call\|>", re.S)

    def __init__(self, tools=None):
        self.tools = tools
        self.buf = ""

    def feed(self, text):
        """Streaming: text passes through (the harmony reasoning parser routes
        channels); calls are read from the whole reply by :meth:`parse`."""
        return text, []

    def flush(self):
        return "", []

    def _call(self, m):
        args = _loads(m.group(2).strip())
        return ToolCall(m.group(1), args if isinstance(args, dict) else {"input": m.group(2)})

    def parse(self, text):
        calls = [self._call(m) for m in self.PAT.finditer(text)]
        content = self.PAT.sub("", text) if calls else text
        return content, calls


TOOL_FORMATS = {
    "json": JSONToolParser, "hermes": JSONToolParser, "qwen3": JSONToolParser,
    "xml_function": XMLFunctionToolParser, "nemotron": NemotronToolParser, "qwen3_5": Qwen35ToolParser,
    "mimo_v2": MiMoV2ToolParser, "glm4": GLM4ToolParser, "glm5": GLM5ToolParser, "flint": FlintToolParser,
    "gemma": GemmaToolParser, "gemma4": Gemma4ToolParser, "kimi_k2": KimiK2ToolParser,
    "minimax_m2": MiniMaxM2ToolParser, "atem": ATEMToolParser, "mistral": MistralToolParser,
    "llama3": Llama3ToolParser, "lfm2": PythonicToolParser, "pythonic": PythonicToolParser,
    "gpt_oss": HarmonyToolParser, "harmony": HarmonyToolParser,
}

# model_type -> format, for configurations that name no format
# (MLXLMCommon/Tool/ToolCallFormatInference.swift)
FORMAT_BY_MODEL_TYPE = {
    "qwen3_5": "qwen3_5", "qwen3_5_moe": "qwen3_5", "qwen3_next": "xml_function", "nemotron_h": "nemotron",
    "glm4": "glm4", "glm4_moe": "glm4", "gemma": "gemma", "gemma2": "gemma", "gemma3": "gemma",
    "gemma3_text": "gemma", "gemma4": "gemma4", "gemma4_text": "gemma4", "kimi_k2": "kimi_k2",
    "minimax": "minimax_m2", "mistral": "mistral", "mistral3": "mistral", "llama": "llama3", "lfm2": "lfm2",
    "lfm2_moe": "lfm2", "gpt_oss": "harmony", "mimo": "mimo_v2", "mimo_v2_flash": "mimo_v2",
}


def infer_tool_format(model_type: str | None) -> str:
    return FORMAT_BY_MODEL_TYPE.get(model_type or "", "json")
