"""Guided (grammar-constrained) generation.

Two native engines: a pushdown (context-free) matcher over EBNF rules
(csrc/host/grammar_pda.cpp; :class:`CfgConstraint`, the default for JSON
objects, JSON schemas and EBNF grammars - recursion is kept, not unrolled)
and a byte-level lazily determinised regex automaton (csrc/host/grammar.cpp;
:class:`GrammarConstraint`, for regex requests). Front ends of the regex
engine:
  * :func:`json_schema_to_regex` - objects (properties in declaration order,
    required / optional), arrays (min/max items), strings (enum, const,
    pattern, min/max length), integers, numbers, booleans, null, anyOf / oneOf,
    ``$ref`` to ``$defs``; recursion and free-form JSON are unrolled to a
    bounded nesting depth;
  * :func:`ebnf_to_regex` - GBNF-style rules ``name ::= alternatives`` with
    quoted literals, character classes, grouping and ``* + ?``; recursive rules
    are unrolled to a bounded depth;
  * regex directly.
:class:`GrammarConstraint` is the per-request token constraint the engine's
sampler consumes (allowed-token mask per step, commit, rollback,
termination). Parity: MLXGuidedGeneration/GuidedGenerationLoop.swift:21-611,
XGrammarBridge.swift (``GrammarConstraint`` :184, ``computeMask`` :515,
``commitToken`` :560, ``rollback`` :698).
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np

_LIBDIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib")
if _LIBDIR not in sys.path:
    sys.path.insert(0, _LIBDIR)
import _b200host  # noqa: E402

WS = r"[ \n]?"  # whitespace policy between JSON tokens
STRING_CHAR = r'([^"\\\x00-\x1f]|\\["\\/bfnrt])'
JSON_STRING = '"' + STRING_CHAR + '*"'
JSON_INT = r"-?(0|[1-9][0-9]{0,15})"
JSON_NUM = JSON_INT + r"(\.[0-9]{1,16})?([eE][+-]?[0-9]{1,3})?"
JSON_BOOL = r"(true|false)"
JSON_NULL = r"null"


def _esc(s: str) -> str:
    out = []
    for ch in s:
        if ch in r"\.^$|?*+()[]{}":
            out.append("\\" + ch)
        elif ch == "\n":
            out.append("\\n")
        else:
            out.append(ch)
    return "".join(out)


def _json_literal(v) -> str:
    return _esc(json.dumps(v))


def any_json(depth: int = 2) -> str:
    scalar = f"({JSON_STRING}|{JSON_NUM}|{JSON_BOOL}|{JSON_NULL})"
    if depth <= 0:
        return scalar
    inner = any_json(depth - 1)
    arr = rf"\[{WS}({inner}({WS},{WS}{inner}){{0,16}})?{WS}\]"
    obj = rf"\{{{WS}({JSON_STRING}{WS}:{WS}{inner}({WS},{WS}{JSON_STRING}{WS}:{WS}{inner}){{0,16}})?{WS}\}}"
    return f"({scalar}|{arr}|{obj})"


def json_schema_to_regex(schema, defs=None, depth: int = 4) -> str:
    if isinstance(schema, str):
        schema = json.loads(schema)
    defs = defs if defs is not None else schema.get("$defs", schema.get("definitions", {}))
    if depth < 0:
        return any_json(0)
    if "$ref" in schema:
        name = schema["$ref"].split("/")[-1]
        return json_schema_to_regex(defs[name], defs, depth - 1)
    if "const" in schema:
        return _json_literal(schema["const"])
    if "enum" in schema:
        return "(" + "|".join(_json_literal(v) for v in schema["enum"]) + ")"
    for key in ("anyOf", "oneOf"):
        if key in schema:
            return "(" + "|".join(json_schema_to_regex(s, defs, depth) for s in schema[key]) + ")"
    t = schema.get("type")
    if isinstance(t, list):
        return "(" + "|".join(json_schema_to_regex({**schema, "type": x}, defs, depth) for x in t) + ")"
    if t == "object" or (t is None and "properties" in schema):
        props = schema.get("properties", {})
        if not props:
            return any_json(min(depth, 2)) if t is None else rf"\{{{WS}({JSON_STRING}{WS}:{WS}{any_json(1)}" \
                rf"({WS},{WS}{JSON_STRING}{WS}:{WS}{any_json(1)}){{0,16}})?{WS}\}}"
        required = set(schema.get("required", list(props)))
        parts = []
        for name, sub in props.items():
            kv = f'"{_esc(name)}"{WS}:{WS}{json_schema_to_regex(sub, defs, depth - 1)}'
            parts.append((kv, name in required))
        # properties in declaration order; a comma precedes every emitted property but the first
        body = ""
        first_emitted_possible = True
        for i, (kv, req) in enumerate(parts):
            if i == 0:
                piece = kv
            else:
                piece = f"{WS},{WS}{kv}" if not first_emitted_possible else f"({WS},{WS})?{kv}"
            body += piece if req else f"({piece})?"
            if req:
                first_emitted_possible = False
        return rf"\{{{WS}{body}{WS}\}}"
    if t == "array":
        item = json_schema_to_regex(schema.get("items", {}), defs, depth - 1)
        lo = int(schema.get("minItems", 0))
        hi = schema.get("maxItems")
        if hi is None:
            rest = f"({WS},{WS}{item})*"
        else:
            rest = f"({WS},{WS}{item}){{0,{max(0, int(hi) - 1)}}}"
        if lo > 0:
            rest_min = "".join(f"{WS},{WS}{item}" for _ in range(lo - 1))
            tail = f"({WS},{WS}{item})*" if hi is None else f"({WS},{WS}{item}){{0,{max(0, int(hi) - lo)}}}"
            return rf"\[{WS}{item}{rest_min}{tail}{WS}\]"
        return rf"\[{WS}({item}{rest})?{WS}\]"
    if t == "string":
        if "pattern" in schema:
            return '"' + schema["pattern"].lstrip("^").rstrip("$") + '"'
        fmt = schema.get("format")
        if fmt == "date":
            return r'"[0-9]{4}-[0-9]{2}-[0-9]{2}"'
        lo, hi = schema.get("minLength"), schema.get("maxLength")
        if lo is not None or hi is not None:
            return '"' + STRING_CHAR + "{" + f"{int(lo or 0)},{'' if hi is None else int(hi)}" + '}"'
        return JSON_STRING
    if t == "integer":
        return JSON_INT
    if t == "number":
        return JSON_NUM
    if t == "boolean":
        return JSON_BOOL
    if t == "null":
        return JSON_NULL
    return any_json(min(depth, 2))


# ----------------------------------------------------------------------------- EBNF
_TOKEN = re.compile(r'\s*(::=|\||\(|\)|\*|\+|\?|"(?:[^"\\]|\\.)*"|\[(?:[^\]\\]|\\.)*\]|[A-Za-z_][\w-]*)')


def ebnf_to_regex(grammar: str, root: str = "root", depth: int = 6) -> str:
    rules = {}
    for line in re.split(r"\n(?=\s*[A-Za-z_][\w-]*\s*::=)", grammar.strip()):
        if "::=" not in line:
            continue
        name, body = line.split("::=", 1)
        rules[name.strip()] = body.strip()

    def expand(name, d):
        if d < 0:
            return "(?!)" if False else "[^\\x00-\\xff]"  # unreachable branch: matches nothing
        toks = [m.group(1) for m in _TOKEN.finditer(rules[name])]
        out = []
        for t in toks:
            if t.startswith('"'):
                out.append(_esc(json.loads(t)))
            elif t.startswith("["):
                out.append(t)
            elif t in ("|", "(", ")", "*", "+", "?"):
                out.append(t)
            else:
                out.append("(" + expand(t, d - 1) + ")")
        return "".join(out)

    return expand(root, depth)


# ----------------------------------------------------------------------------- vocab
def token_bytes(tokenizer, vocab_size: int) -> list[bytes]:
    """Byte string of every token id (empty for special tokens)."""
    if hasattr(tokenizer, "get_vocab_strings") and type(tokenizer).__name__ == "ByteTokenizer":
        out = []
        for i in range(vocab_size):
            out.append(bytes([i]) if i < 256 else b"")
        return out
    tok = getattr(tokenizer, "tok", tokenizer)
    special = set(getattr(tok, "all_special_ids", []) or [])
    out = []
    try:
        pieces = tok.convert_ids_to_tokens(list(range(min(vocab_size, len(tok)))))
    except Exception:
        pieces = None
    bdec = _gpt2_byte_decoder()
    for i in range(vocab_size):
        if i in special or pieces is None or i >= len(pieces) or pieces[i] is None:
            out.append(b"")
            continue
        p = pieces[i]
        if p.startswith("<0x") and p.endswith(">") and len(p) == 6:  # sentencepiece byte fallback
            out.append(bytes([int(p[3:5], 16)]))
        elif "▁" in p:
            out.append(p.replace("▁", " ").encode("utf-8"))
        elif all(c in bdec for c in p):
            out.append(bytes(bdec[c] for c in p))
        else:
            out.append(p.encode("utf-8"))
    return out


def _gpt2_byte_decoder():
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return {chr(c): b for b, c in zip(bs, cs)}


class GrammarVocabulary:
    """Shared per-tokenizer trie (build once, reuse for every request)."""

    def __init__(self, tokenizer, vocab_size: int, eos_ids):
        self.size = vocab_size
        self.native = _b200host.GrammarVocab(token_bytes(tokenizer, vocab_size), sorted(int(e) for e in eos_ids))


class GrammarConstraint:
    """Per-request constraint consumed by the engine's sampler."""

    def __init__(self, vocab: GrammarVocabulary, regex: str):
        self.vocab = vocab
        self.regex = regex
        self.m = _b200host.GrammarMatcher(vocab.native, regex)
        self.n_committed = 0

    @classmethod
    def from_json_schema(cls, vocab, schema):
        return cls(vocab, json_schema_to_regex(schema))

    @classmethod
    def from_ebnf(cls, vocab, grammar, root="root"):
        return cls(vocab, ebnf_to_regex(grammar, root))

    @classmethod
    def json_object(cls, vocab):
        return cls(vocab, WS + any_json(3) + WS)

    def allowed_mask(self, V: int) -> np.ndarray:
        words = self.m.mask()
        bits = np.unpackbits(words.view(np.uint8), bitorder="little")[:V].astype(bool)
        if bits.shape[0] < V:
            bits = np.pad(bits, (0, V - bits.shape[0]))
        return bits

    def commit(self, tok: int):
        if not self.m.accept_token(int(tok)):
            raise ValueError(f"token {tok} violates the grammar")
        self.n_committed += 1

    def rollback(self, n: int):
        self.m.rollback(int(n))
        self.n_committed -= n

    def is_terminated(self) -> bool:
        return self.m.is_terminated()

    def forced_prefix(self) -> bytes:
        return self.m.forced_prefix()


def constraint_factory(vocab: GrammarVocabulary):
    """OpenAI ``response_format`` -> constraint (server hook)."""

    def make(rf: dict):
        t = rf.get("type")
        if t == "json_object":
            return CfgConstraint.json_object(vocab)
        if t == "json_schema":
            js = rf.get("json_schema", {})
            return CfgConstraint.from_json_schema(vocab, js.get("schema", js))
        if t == "regex":
            return GrammarConstraint(vocab, rf["regex"])
        if t == "grammar":
            return CfgConstraint.from_ebnf(vocab, rf["grammar"], rf.get("root", "root"))
        if t == "structural_tag":
            return CfgConstraint.from_structural_tag(vocab, rf["structures"], rf["triggers"])
        return None

    return make


# ----------------------------------------------------------------------------- context-free front ends
# The pushdown engine (csrc/host/grammar_pda.cpp) takes EBNF rules directly, so
# recursive schemas and grammars need no unrolling.
JSON_EBNF_BASE = r'''
ws ::= [ \n]?
json-char ::= [^"\\\x00-\x1f] | "\\" ( ["\\/bfnrt] | "u" [0-9a-fA-F]{4} )
json-string ::= "\"" json-char* "\""
json-int ::= "-"? ( "0" | [1-9] [0-9]{0,15} )
json-number ::= json-int ( "." [0-9]{1,16} )? ( [eE] [+-]? [0-9]{1,3} )?
json-bool ::= "true" | "false"
json-null ::= "null"
json-value ::= json-object | json-array | json-string | json-number | json-bool | json-null
json-object ::= "{" ws ( json-string ws ":" ws json-value ( ws "," ws json-string ws ":" ws json-value )* )? ws "}"
json-array ::= "[" ws ( json-value ( ws "," ws json-value )* )? ws "]"
'''


def _ebnf_lit(s: str) -> str:
    """A quoted EBNF literal of the text s."""
    out = ['"']
    for ch in s:
        o = ord(ch)
        if ch in '"\\':
            out.append("\\" + ch)
        elif o < 0x20:
            out.append(f"\\x{o:02x}")
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


_RX_ESC = {"d": "[0-9]", "w": "[A-Za-z0-9_]", "s": "[ \\t\\n\\r]", "D": "[^0-9]", "W": "[^A-Za-z0-9_]",
           "S": "[^ \\t\\n\\r]", "n": '"\\n"', "t": '"\\t"', "r": '"\\r"'}


def regex_to_ebnf(rx: str) -> str:
    """The EBNF body of a (JSON-schema ``pattern`` style) regular expression:
    literals become quoted strings, classes / groups / alternation /
    quantifiers carry over, anchors are dropped."""
    out, i, n = [], 0, len(rx)
    while i < n:
        c = rx[i]
        if c in "^$" and (i == 0 or i == n - 1):
            i += 1
        elif c == "[":
            j = i + 1
            if j < n and rx[j] == "^":
                j += 1
            if j < n and rx[j] == "]":
                j += 1
            while j < n and rx[j] != "]":
                j += 2 if rx[j] == "\\" else 1
            out.append(rx[i:j + 1])
            i = j + 1
        elif c == "\\" and i + 1 < n:
            e = rx[i + 1]
            out.append(_RX_ESC.get(e, _ebnf_lit(e)))
            i += 2
        elif c in "()|*+?":
            out.append(c)
            i += 1
        elif c == "{":
            j = rx.index("}", i)
            out.append(rx[i:j + 1])
            i = j + 1
        elif c == ".":
            out.append("[^\\n]")
            i += 1
        else:
            out.append(_ebnf_lit(c))
            i += 1
    return " ".join(out) if out else '""'


class _SchemaEbnf:
    def __init__(self, schema: dict):
        self.root_schema = schema
        self.defs = schema.get("$defs", schema.get("definitions", {}))
        self.rules: dict[str, str] = {}
        self.ref_rules: dict[str, str] = {}
        self.n = 0

    def new(self, hint: str) -> str:
        self.n += 1
        return f"s{self.n}-{re.sub(r'[^A-Za-z0-9]', '', hint)[:16] or 'x'}"

    def rule(self, schema, hint="v") -> str:
        """Name of a rule matching `schema`."""
        if isinstance(schema, bool):
            return "json-value" if schema else self._never()
        if "$ref" in schema:
            ref = schema["$ref"]
            if ref in self.ref_rules:
                return self.ref_rules[ref]
            name = self.new(ref.split("/")[-1])
            self.ref_rules[ref] = name  # registered before the body: recursion refers to it
            target = self.root_schema if ref == "#" else self.defs[ref.split("/")[-1]]
            self.rules[name] = self.rule(target, ref.split("/")[-1])
            return name
        body = self.body(schema, hint)
        name = self.new(hint)
        self.rules[name] = body
        return name

    def _never(self) -> str:
        self.rules.setdefault("never", "[^\\x00-\\xff]")  # an empty byte class
        return "never"

    def body(self, schema: dict, hint: str) -> str:
        if "const" in schema:
            return _ebnf_lit(json.dumps(schema["const"]))
        if "enum" in schema:
            return " | ".join(_ebnf_lit(json.dumps(v)) for v in schema["enum"])
        for key in ("anyOf", "oneOf"):
            if key in schema:
                return " | ".join(self.rule(s, hint) for s in schema[key])
        if "allOf" in schema:  # merged shallowly: properties and required of every part
            merged: dict = {}
            for part in schema["allOf"]:
                part = self.defs[part["$ref"].split("/")[-1]] if "$ref" in part else part
                for k, v in part.items():
                    if k == "properties":
                        merged.setdefault("properties", {}).update(v)
                    elif k == "required":
                        merged.setdefault("required", []).extend(v)
                    else:
                        merged[k] = v
            return self.body(merged, hint)
        t = schema.get("type")
        if isinstance(t, list):
            return " | ".join(self.rule({**schema, "type": x}, hint) for x in t)
        if t == "object" or (t is None and "properties" in schema):
            return self.obj(schema, hint)
        if t == "array" or (t is None and "items" in schema):
            return self.arr(schema, hint)
        if t == "string":
            return self.string(schema)
        if t == "integer":
            return "json-int"
        if t == "number":
            return "json-number"
        if t == "boolean":
            return "json-bool"
        if t == "null":
            return "json-null"
        return "json-value"

    def obj(self, schema, hint):
        props = schema.get("properties", {})
        extra = schema.get("additionalProperties", not props)
        if not props:
            if extra is False:
                return '"{" ws "}"'
            val = "json-value" if extra in (True, None) or extra == {} else self.rule(extra, hint + "v")
            kv = f"json-string ws \":\" ws {val}"
            return f'"{{" ws ( {kv} ( ws "," ws {kv} )* )? ws "}}"'
        required = set(schema.get("required", []))
        parts = [(f"{_ebnf_lit(json.dumps(name))} ws \":\" ws {self.rule(sub, name)}", name in required)
                 for name, sub in props.items()]
        # declaration order; a comma precedes every emitted property but the first
        body, first_possible = "", True
        for i, (kv, req) in enumerate(parts):
            if i == 0:
                piece = kv
            elif first_possible:
                piece = f'( ws "," ws )? {kv}'
            else:
                piece = f'ws "," ws {kv}'
            body += f" {piece}" if req else f" ( {piece} )?"
            if req:
                first_possible = False
        return f'"{{" ws{body} ws "}}"'

    def arr(self, schema, hint):
        item = self.rule(schema.get("items", {}), hint + "i")
        lo = int(schema.get("minItems", 0))
        hi = schema.get("maxItems")
        more = f'ws "," ws {item}'
        if hi is not None and int(hi) == 0:
            return '"[" ws "]"'
        if lo > 0:
            rest = f"( {more} ){{{lo - 1},{'' if hi is None else int(hi) - 1}}}"
            return f'"[" ws {item} {rest} ws "]"'
        rest = f"( {more} )*" if hi is None else f"( {more} ){{0,{int(hi) - 1}}}"
        return f'"[" ws ( {item} {rest} )? ws "]"'

    def string(self, schema):
        if "pattern" in schema:
            return f'"\\"" ( {regex_to_ebnf(schema["pattern"])} ) "\\""'
        fmt = schema.get("format")
        if fmt == "date":
            return '"\\"" [0-9]{4} "-" [0-9]{2} "-" [0-9]{2} "\\""'
        if fmt == "date-time":
            return ('"\\"" [0-9]{4} "-" [0-9]{2} "-" [0-9]{2} "T" [0-9]{2} ":" [0-9]{2} ":" [0-9]{2} '
                    '( "." [0-9]{1,9} )? ( "Z" | [+-] [0-9]{2} ":" [0-9]{2} ) "\\""')
        if fmt == "uuid":
            return ('"\\"" [0-9a-fA-F]{8} "-" [0-9a-fA-F]{4} "-" [0-9a-fA-F]{4} "-" [0-9a-fA-F]{4} "-" '
                    '[0-9a-fA-F]{12} "\\""')
        lo, hi = schema.get("minLength"), schema.get("maxLength")
        if lo is not None or hi is not None:
            return f'"\\"" json-char{{{int(lo or 0)},{"" if hi is None else int(hi)}}} "\\""'
        return "json-string"


def json_schema_to_ebnf(schema) -> str:
    """EBNF (root rule ``root``) of the JSON documents a schema admits, with
    ``$ref`` recursion kept as rule references (no depth bound)."""
    if isinstance(schema, str):
        schema = json.loads(schema)
    conv = _SchemaEbnf(schema)
    top = conv.rule(schema, "root")
    lines = [f"root ::= ws {top} ws"] + [f"{k} ::= {v}" for k, v in conv.rules.items()]
    return "\n".join(lines) + "\n" + JSON_EBNF_BASE


_COMPILED: "dict[tuple, object]" = {}
_COMPILED_MAX = 64


def compiled_grammar(vocab: GrammarVocabulary, grammar: str, root: str = "root"):
    """The grammar compiled against `vocab`, shared by every request that uses
    it (its per-state token classes are computed once); a small LRU."""
    key = (id(vocab.native), grammar, root)
    c = _COMPILED.pop(key, None)
    if c is None:
        c = _b200host.CfgGrammar(vocab.native, grammar, root)
    _COMPILED[key] = c
    while len(_COMPILED) > _COMPILED_MAX:
        _COMPILED.pop(next(iter(_COMPILED)))
    return c


class CfgConstraint(GrammarConstraint):
    """Per-request constraint on the pushdown (context-free) engine: same
    interface as :class:`GrammarConstraint`."""

    def __init__(self, vocab: GrammarVocabulary, grammar: str, root: str = "root"):
        self.vocab = vocab
        self.grammar = grammar
        self.m = _b200host.CfgMatcher(compiled_grammar(vocab, grammar, root))
        self.n_committed = 0

    @classmethod
    def from_json_schema(cls, vocab, schema):
        return cls(vocab, json_schema_to_ebnf(schema))

    @classmethod
    def from_ebnf(cls, vocab, grammar, root="root"):
        return cls(vocab, grammar, root)

    @classmethod
    def json_object(cls, vocab):
        return cls(vocab, "root ::= ws json-object ws\n" + JSON_EBNF_BASE)

    @classmethod
    def from_structural_tag(cls, vocab, structures, triggers):
        return cls(vocab, structural_tag_to_ebnf(structures, triggers))


# ----------------------------------------------------------------------------- structural tags
def _byte_class(bs) -> str:
    """EBNF byte class of the byte values `bs` (sorted ranges, \\xHH escapes)."""
    bs = sorted(set(bs))
    parts, i = [], 0
    while i < len(bs):
        j = i
        while j + 1 < len(bs) and bs[j + 1] == bs[j] + 1:
            j += 1
        parts.append(f"\\x{bs[i]:02x}" if i == j else f"\\x{bs[i]:02x}-\\x{bs[j]:02x}")
        i = j + 1
    return "[" + "".join(parts) + "]"


def structural_tag_to_ebnf(structures: list[dict], triggers: list[str]) -> str:
    """EBNF of free text in which every occurrence of a trigger starts a tagged
    call: ``begin`` (which starts with the trigger), a JSON document of the
    tag's ``schema``, then ``end``; free text resumes after it. The free text
    is the Aho-Corasick automaton of the triggers written as right-linear
    rules (one per automaton state; tail calls keep the stack flat). Triggers
    are ASCII. Parity: the structural tags of xgrammar
    (Libraries/MLXCXGrammar/xgrammar/cpp/structural_tag.cc) as used for tool
    calls."""
    if not triggers:
        raise ValueError("structural tag: at least one trigger")
    for t in triggers:
        if not t or any(ord(c) > 0x7F for c in t):
            raise ValueError(f"structural tag: trigger {t!r} must be non-empty ASCII")
    by_trigger: dict[str, list[dict]] = {t: [] for t in triggers}
    for s in structures:
        trig = next((t for t in triggers if s["begin"].startswith(t)), None)
        if trig is None:
            raise ValueError(f"structural tag: begin {s['begin']!r} starts with no trigger")
        by_trigger[trig].append(s)
    # Aho-Corasick over the trigger bytes
    goto: list[dict[int, int]] = [{}]
    out: list[str | None] = [None]
    for t in triggers:
        q = 0
        for b in t.encode():
            if b not in goto[q]:
                goto.append({})
                out.append(None)
                goto[q][b] = len(goto) - 1
            q = goto[q][b]
        out[q] = t
    fail = [0] * len(goto)
    order = list(goto[0].values())
    i = 0
    while i < len(order):
        q = order[i]
        i += 1
        for b, r in goto[q].items():
            f = fail[q]
            while f and b not in goto[f]:
                f = fail[f]
            fail[r] = goto[f][b] if b in goto[f] and goto[f][b] != r else 0
            if out[r] is None and out[fail[r]] is not None:
                out[r] = out[fail[r]]
            order.append(r)

    def step(q, b):
        while q and b not in goto[q]:
            q = fail[q]
        return goto[q].get(b, 0)

    conv = _SchemaEbnf({})
    lines = ["root ::= text-0"]
    for q in range(len(goto)):
        if out[q] is not None:  # a trigger just completed: one of its tags follows
            trig = out[q]
            alts = []
            for s in by_trigger[trig]:
                body = conv.rule(s.get("schema", {}), "tag")
                rest = s["begin"][len(trig):]
                alts.append(" ".join(x for x in (_ebnf_lit(rest) if rest else "", f"ws {body} ws",
                                                _ebnf_lit(s["end"]), "text-0") if x))
            lines.append(f"text-{q} ::= " + (" | ".join(alts) if alts else '[^\\x00-\\xff]'))
            continue
        targets: dict[int, list[int]] = {}
        for b in range(256):
            targets.setdefault(step(q, b), []).append(b)
        alts = ['""'] + [f"{_byte_class(bs)} text-{r}" for r, bs in sorted(targets.items())]
        lines.append(f"text-{q} ::= " + " | ".join(alts))
    lines += [f"{k} ::= {v}" for k, v in conv.rules.items()]
    return "\n".join(lines) + "\n" + JSON_EBNF_BASE
