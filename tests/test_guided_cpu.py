"""Grammar engine + guided generation through the engine (CPU)."""
import json
import re

import numpy as np
import pytest
import torch

from mlx_swift_lm_b200.api.guided import (GrammarConstraint, GrammarVocabulary, ebnf_to_regex,
                                          json_schema_to_regex)
from mlx_swift_lm_b200.api.tokenizer import ByteTokenizer


@pytest.fixture(scope="module")
def vocab():
    tok = ByteTokenizer(512)
    return tok, GrammarVocabulary(tok, 512, [tok.eos_token_id])


def _drive(c, text, eos):
    for ch in text.encode():
        assert c.allowed_mask(512)[ch], (text, chr(ch))
        c.commit(ch)
    assert c.allowed_mask(512)[eos]
    c.commit(eos)
    assert c.is_terminated()


def test_regex_masks_and_rollback(vocab):
    tok, v = vocab
    c = GrammarConstraint(v, r"(yes|no)!")
    m = c.allowed_mask(512)
    assert set(np.nonzero(m)[0]) == {ord("y"), ord("n")}
    c.commit(ord("y"))
    assert set(np.nonzero(c.allowed_mask(512))[0]) == {ord("e")}
    c.rollback(1)
    assert c.allowed_mask(512)[ord("n")]
    with pytest.raises(ValueError):
        c.commit(ord("x"))


def test_json_schema_regex_accepts_valid_documents(vocab):
    tok, v = vocab
    schema = {"type": "object", "properties": {
        "name": {"type": "string"}, "age": {"type": "integer"}, "tags": {"type": "array", "items": {"enum": ["a", "b"]}},
        "ok": {"type": "boolean"}}, "required": ["name", "age"]}
    rx = json_schema_to_regex(schema)
    for doc in [{"name": "x", "age": 3}, {"name": "y z", "age": -12, "tags": ["a", "b"], "ok": True}]:
        s = json.dumps(doc, separators=(",", ":"))
        assert re.fullmatch(rx, s), s
        _drive(GrammarConstraint(v, rx), s, tok.eos_token_id)
    assert not re.fullmatch(rx, json.dumps({"age": 3}))


def test_ebnf_lowering(vocab):
    tok, v = vocab
    g = 'root ::= greeting " " name\ngreeting ::= "hi" | "hello"\nname ::= [a-z]+'
    rx = ebnf_to_regex(g)
    assert re.fullmatch(rx, "hello bob") and not re.fullmatch(rx, "hey bob")
    _drive(GrammarConstraint(v, rx), "hi al", tok.eos_token_id)


def test_guided_generation_through_engine():
    from mlx_swift_lm_b200.api.container import ModelContainer
    from mlx_swift_lm_b200.engine.engine import EngineConfig
    from mlx_swift_lm_b200.engine.types import Request, SamplingParams
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    cfg = tiny_qwen3()
    cfg.vocab_size = 512
    c = ModelContainer.random(cfg, "cpu", torch.float32, seed=3, std=0.2,
                              engine_config=EngineConfig(max_model_len=512, use_cuda_graphs=False))
    v = GrammarVocabulary(c.tokenizer, 512, [c.tokenizer.eos_token_id])
    schema = {"type": "object", "properties": {"answer": {"enum": ["red", "green"]}, "n": {"type": "integer"}},
              "required": ["answer", "n"]}
    con = GrammarConstraint.from_json_schema(v, schema)
    st = c.engine.submit(Request(prompt_tokens=c.encode("color?"), max_tokens=40,
                                 sampling=SamplingParams(temperature=0.7, seed=5), token_constraint=con))
    c.engine.run_until_idle()
    text = c.decode([t for t in st.tokens() if t < 256])
    obj = json.loads(text)
    assert obj["answer"] in ("red", "green") and isinstance(obj["n"], int)
