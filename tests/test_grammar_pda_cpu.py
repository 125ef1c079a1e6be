"""Pushdown (context-free) grammar engine: EBNF with unbounded recursion,
JSON schemas with recursive $ref, token masks equal to brute force over a
multi-byte vocabulary, rollback / forced prefix, refusal of left recursion,
and constrained generation through the engine."""
import json
import random

import numpy as np
import pytest
import torch

from mlx_swift_lm_b200.api.guided import (JSON_EBNF_BASE, CfgConstraint, GrammarVocabulary, json_schema_to_ebnf,
                                          regex_to_ebnf)
from mlx_swift_lm_b200.api.tokenizer import ByteTokenizer

JSON_G = "root ::= ws json-value ws\n" + JSON_EBNF_BASE


class _Tok:
    """Bytes 0-255 plus multi-byte pieces; id 300 is EOS."""
    PIECES = [b'{"', b'":', b'",', b'"}', b'true', b'false', b'null', b'[', b'],', b'ab', b'abc"', b'12', b'{"a":',
              b'"b"', b' [', b'\\"', b'\\u00', b'e+', b'0.5', b']}', b'}}', b'::', b'\xc3\xa9']

    def __init__(self):
        self.eos_token_id = 300

    def pieces(self):
        out = [bytes([i]) for i in range(256)] + self.PIECES
        return out + [b""] * (301 - len(out))


@pytest.fixture(scope="module")
def mb_vocab():
    t = _Tok()
    import mlx_swift_lm_b200.api.guided as g
    v = GrammarVocabulary.__new__(GrammarVocabulary)
    v.size = 301
    v.native = g._b200host.GrammarVocab(t.pieces(), [300])
    return t, v


def _allowed(c, V):
    return set(np.nonzero(c.allowed_mask(V))[0].tolist())


def _brute(c, V):
    ok = set()
    for i in range(V):
        if c.m.accept_token(i):
            ok.add(i)
            c.m.rollback(1)
    return ok


def test_json_documents_any_depth(mb_vocab):
    t, v = mb_vocab
    deep = "[" * 40 + "1" + "]" * 40
    for doc in ['{"a": [1, {"b": [true, null, "x\\"y"]}, []], "c": -3.5e+2}', deep, '"\\u00e9"', " null "]:
        c = CfgConstraint(v, JSON_G)
        for ch in doc.encode():
            assert ch in _allowed(c, 301), (doc, chr(ch))
            c.commit(ch)
        assert 300 in _allowed(c, 301)
        c.commit(300)
        assert c.is_terminated()
    c = CfgConstraint(v, JSON_G)
    for ch in b'{"a" 1':
        if ch not in _allowed(c, 301):
            break
        c.commit(ch)
    else:
        raise AssertionError("accepted a missing colon")


def test_masks_equal_brute_force(mb_vocab):
    t, v = mb_vocab
    rng = random.Random(0)
    docs = ['{"a": [1, {"b": [true, null, "xy"]}, []], "c": -3.5}', '[{"k": "v\\n"}, 0.5, false]']
    for doc in docs:
        c = CfgConstraint(v, JSON_G)
        for k, ch in enumerate(doc.encode()):
            if k % 3 == 0 or rng.random() < 0.3:
                assert _allowed(c, 301) == _brute(c, 301), (doc[:k], k)
            c.commit(ch)


def test_recursive_schema(mb_vocab):
    t, v = mb_vocab
    schema = {"$defs": {"node": {"type": "object", "properties": {
        "name": {"type": "string", "maxLength": 8}, "kids": {"type": "array", "items": {"$ref": "#/$defs/node"}}},
        "required": ["name"]}}, "$ref": "#/$defs/node"}
    g = json_schema_to_ebnf(schema)

    def tree(d):
        return {"name": f"n{d}", "kids": [tree(d - 1)] if d else []}

    ok = json.dumps(tree(9))  # deeper than any unrolled regex
    c = CfgConstraint(v, g)
    for ch in ok.encode():
        assert ch in _allowed(c, 301), chr(ch)
        c.commit(ch)
    assert c.m.is_accepting()
    for bad in ['{"kids": []}', '{"name": "waytoolongname"}', '{"name": "a", "kids": [1]}']:
        c = CfgConstraint(v, g)
        good = True
        for ch in bad.encode():
            if ch not in _allowed(c, 301):
                good = False
                break
            c.commit(ch)
        assert not good or not c.m.is_accepting(), bad


def test_schema_features(mb_vocab):
    t, v = mb_vocab
    schema = {"type": "object", "properties": {
        "id": {"type": "string", "format": "uuid"}, "when": {"type": "string", "format": "date"},
        "code": {"type": "string", "pattern": "^[A-Z]{2}-\\d{3}$"}, "n": {"type": "integer"},
        "x": {"anyOf": [{"type": "number"}, {"type": "null"}]}, "tags": {"type": "array", "items": {"enum": ["a", "b"]},
                                                                          "minItems": 1, "maxItems": 2},
        "c": {"const": {"k": [1, 2]}}}, "required": ["id", "code", "tags"]}
    g = json_schema_to_ebnf(schema)
    good = {"id": "123e4567-e89b-12d3-a456-426614174000", "when": "2026-12-02", "code": "AB-123", "n": -4,
            "x": None, "tags": ["b", "a"], "c": {"k": [1, 2]}}
    for doc in [json.dumps(good), json.dumps({k: good[k] for k in ("id", "code", "tags")})]:
        c = CfgConstraint(v, g)
        for ch in doc.encode():
            assert ch in _allowed(c, 301), (doc, chr(ch))
            c.commit(ch)
        assert c.m.is_accepting()
    for bad in [dict(good, code="ab-123"), dict(good, tags=[]), dict(good, tags=["a", "b", "a"])]:
        c = CfgConstraint(v, g)
        doc = json.dumps(bad)
        accepted = all(ch in _allowed(c, 301) and (c.commit(ch) or True) for ch in doc.encode())
        assert not (accepted and c.m.is_accepting()), doc


def test_ebnf_rollback_forced_prefix_and_left_recursion(mb_vocab):
    t, v = mb_vocab
    g = '''
    # a greeting, then a list of names
    root ::= greet ": " names "."
    greet ::= "hello" | "hi"
    names ::= name ( ", " name ){0,2}
    name ::= [A-Z] [a-z]{1,5}
    '''
    c = CfgConstraint(v, g)
    for ch in b"hello: Al, Bo":
        c.commit(ch)
    c.rollback(4)  # back to "hello: Al"
    assert ord(",") in _allowed(c, 301) and ord(".") in _allowed(c, 301)
    c2 = CfgConstraint(v, 'root ::= "prefix-" [0-9]+')
    assert c2.forced_prefix() == b"prefix-"
    with pytest.raises(RuntimeError):
        CfgConstraint(v, 'root ::= root "a" | "b"')
    with pytest.raises(ValueError):
        CfgConstraint(v, 'root ::= undefined-rule')


def test_regex_to_ebnf():
    assert regex_to_ebnf(r"^[A-Z]{2}-\d{3}$") == '[A-Z] {2} "-" [0-9] {3}'


def test_cfg_guided_generation_through_engine():
    from mlx_swift_lm_b200.api.container import ModelContainer
    from mlx_swift_lm_b200.engine.engine import EngineConfig
    from mlx_swift_lm_b200.engine.types import Request, SamplingParams
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    cfg = tiny_qwen3()
    cfg.vocab_size = 512
    c = ModelContainer.random(cfg, "cpu", torch.float32, seed=4, std=0.2,
                              engine_config=EngineConfig(max_model_len=512, use_cuda_graphs=False))
    v = GrammarVocabulary(c.tokenizer, 512, [c.tokenizer.eos_token_id])
    schema = {"$defs": {"t": {"type": "object", "properties": {"v": {"type": "integer"}, "c": {
        "type": "array", "items": {"$ref": "#/$defs/t"}, "maxItems": 1}}, "required": ["v", "c"]}},
        "$ref": "#/$defs/t"}
    con = CfgConstraint.from_json_schema(v, schema)
    st = c.engine.submit(Request(prompt_tokens=c.encode("tree?"), max_tokens=120,
                                 sampling=SamplingParams(temperature=0.8, seed=2), token_constraint=con))
    c.engine.run_until_idle()
    toks = st.tokens()
    text = c.decode([t for t in toks if t < 256])
    if toks and toks[-1] == c.tokenizer.eos_token_id:  # finished inside the budget: a full document
        obj = json.loads(text)
        assert isinstance(obj["v"], int) and isinstance(obj["c"], list)
    else:  # budget hit: still a valid prefix of some document
        c2 = CfgConstraint.from_json_schema(v, schema)
        assert c2.m.accept_string(text.encode())


def test_structural_tag(mb_vocab):
    """Free text with tagged tool calls: after the trigger the call must be
    the tag's JSON schema and end string; near-misses of the trigger stay free
    text; long free text keeps a flat stack (tail calls)."""
    from mlx_swift_lm_b200.api.guided import structural_tag_to_ebnf

    t, v = mb_vocab
    schema = {"type": "object", "properties": {"name": {"enum": ["get_weather", "add"]},
                                               "arguments": {"type": "object"}}, "required": ["name", "arguments"]}
    g = structural_tag_to_ebnf([{"begin": "<tool_call>", "schema": schema, "end": "</tool_call>"}], ["<tool_call>"])
    ok = ('Sure <tool> <tool_cal <b> let me check. <tool_call>{"name": "add", "arguments": {"a": 1}}</tool_call>'
          ' and <tool_call>{"name": "get_weather", "arguments": {}}</tool_call> done')
    c = CfgConstraint(v, g)
    for ch in ok.encode():
        assert ch in _allowed(c, 301), (ok, chr(ch))
        c.commit(ch)
        assert c.m.num_stacks <= 8
    assert 300 in _allowed(c, 301)
    for bad in ['x <tool_call>{"name": "rm"', 'x <tool_call>{"name": "add", "arguments": {}}</tool_cal> ']:
        c = CfgConstraint(v, g)
        good = True
        for ch in bad.encode():
            if ch not in _allowed(c, 301):
                good = False
                break
            c.commit(ch)
        assert not good, bad
    c = CfgConstraint(v, g)
    for ch in (b"free text " * 200):
        c.commit(ch)
    assert c.m.num_stacks <= 4
