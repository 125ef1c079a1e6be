"""OpenAI-compatible server over the engine (tiny random model on CPU), plus
the reasoning and tool-call parsers."""
import json

import pytest
import torch

from mlx_swift_lm_b200.api.container import ModelContainer
from mlx_swift_lm_b200.api.parsers import (HarmonyToolParser, JSONObjectToolParser, TaggedJSONToolParser,
                                           ThinkReasoningParser, ToolCall, make_reasoning_parser,
                                           validate_tool_arguments)
from mlx_swift_lm_b200.engine.engine import EngineConfig
from mlx_swift_lm_b200.engine.scheduler import SchedulerConfig
from mlx_swift_lm_b200.models.config import tiny_qwen3


@pytest.fixture(scope="module")
def client():
    from starlette.testclient import TestClient

    from mlx_swift_lm_b200.server.app import OpenAIService, build_app

    cfg = tiny_qwen3()
    cfg.vocab_size = 512
    c = ModelContainer.random(cfg, "cpu", torch.float32, seed=1, std=0.2,
                              engine_config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=8),
                                                         max_model_len=512, use_cuda_graphs=False,
                                                         enable_prefix_cache=True))
    svc = OpenAIService(c, model_name="tiny", tool_parser="hermes", reasoning_parser="qwen3", default_max_tokens=8)
    with TestClient(build_app(svc)) as tc:
        yield tc
    c.engine.shutdown()


def test_health_models_props_metrics(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    props = client.get("/props").json()
    assert "POST /v1/chat/completions" in props["routes"]
    assert "b200lm_requests_total" in client.get("/metrics").text


def test_chat_completion_and_usage(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 6,
                                                   "temperature": 0})
    d = r.json()
    assert r.status_code == 200, d
    assert d["object"] == "chat.completion" and d["usage"]["completion_tokens"] == 6
    assert d["choices"][0]["finish_reason"] == "length"


def test_chat_streaming_sse(client):
    with client.stream("POST", "/v1/chat/completions", json={"messages": [{"role": "user", "content": "yo"}],
                                                              "max_tokens": 5, "stream": True, "temperature": 0,
                                                              "stream_options": {"include_usage": True}}) as r:
        lines = [ln for ln in r.iter_lines() if ln.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    last = json.loads(lines[-2][6:])
    assert last["choices"][0]["finish_reason"] == "length" and last["usage"]["completion_tokens"] == 5


def test_completions_tokenize_detokenize_template(client):
    d = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 4, "temperature": 0}).json()
    assert d["object"] == "text_completion"
    toks = client.post("/tokenize", json={"content": "hello"}).json()["tokens"]
    assert client.post("/detokenize", json={"tokens": toks}).json()["content"] == "hello"
    p = client.post("/apply-template", json={"messages": [{"role": "user", "content": "x"}]}).json()["prompt"]
    assert "<|im_start|>user" in p


def test_responses_store_and_cancel(client):
    d = client.post("/v1/responses", json={"input": "hello", "max_output_tokens": 4}).json()
    assert d["status"] == "completed" and d["output"][0]["type"] == "message"
    g = client.get(f"/v1/responses/{d['id']}").json()
    assert g["id"] == d["id"]
    assert client.get("/v1/responses/nope").status_code == 404


def test_batch_and_embeddings(client):
    d = client.post("/v1/chat/completions/batch", json={"requests": [
        {"messages": [{"role": "user", "content": "a"}], "max_tokens": 3, "temperature": 0},
        {"messages": [{"role": "user", "content": "b"}], "max_tokens": 3, "temperature": 0}]}).json()
    assert len(d["data"]) == 2
    e = client.post("/v1/embeddings", json={"input": ["x", "yz"]}).json()
    assert len(e["data"]) == 2 and abs(sum(v * v for v in e["data"][0]["embedding"]) - 1) < 1e-3


def test_validation_errors(client):
    assert client.post("/v1/chat/completions", json={"messages": []}).status_code == 400
    assert client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                      "temperature": 5}).status_code == 400
    assert client.post("/v1/chat/completions", content=b"{not json").status_code == 400


def test_think_parser_streaming():
    p = ThinkReasoningParser()
    outs = [p.feed(x) for x in ["hel", "lo <th", "ink>rea", "son</th", "ink> done"]]
    r = "".join(o[0] for o in outs) + p.flush()[0]
    c = "".join(o[1] for o in outs)
    assert r == "reason" and c == "hello  done"
    p2 = make_reasoning_parser("deepseek_r1")
    r2, c2 = p2.feed("deep</think>answer")
    assert r2 == "deep" and c2 == "answer"


def test_harmony_reasoning_and_tools():
    p = make_reasoning_parser("harmony")
    r, c = p.feed("<|channel|>analysis<|message|>think hard<|end|><|start|>assistant<|channel|>final<|message|>42")
    assert "think hard" in r and c.endswith("42")
    txt = '<|channel|>commentary to=functions.get_weather <|constrain|>json<|message|>{"city":"Paris"}<|call|>'
    content, calls = HarmonyToolParser().parse(txt)
    assert calls[0].name == "get_weather" and calls[0].arguments == {"city": "Paris"}


def test_tool_parsers():
    p = TaggedJSONToolParser()
    c, calls = p.feed('Sure. <tool_call>{"name": "add", "arguments": {"a": 1}}</tool_call>')
    assert c == "Sure. " and calls[0].name == "add" and calls[0].arguments == {"a": 1}
    c, calls = JSONObjectToolParser().parse('{"name": "f", "parameters": {"x": "y"}}')
    assert calls[0].name == "f"
    c, calls = JSONObjectToolParser("[TOOL_CALLS]").parse('[TOOL_CALLS][{"name": "g", "arguments": {}}]')
    assert calls[0].name == "g"
    tools = [{"type": "function", "function": {"name": "add", "parameters": {
        "type": "object", "properties": {"a": {"type": "integer"}}, "required": ["a", "b"]}}}]
    errs = validate_tool_arguments(ToolCall("add", {"a": "1"}), tools)
    assert any("missing" in e for e in errs) and any("integer" in e for e in errs)
