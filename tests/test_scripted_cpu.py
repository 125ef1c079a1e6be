"""The scripted model drives the real engine: text, stop strings, EOS,
tool-call parsing, all with output known in advance."""
from mlx_swift_lm_b200 import EngineConfig, EngineV2, Request, SchedulerConfig
from mlx_swift_lm_b200.engine.types import SamplingParams
from mlx_swift_lm_b200.testing.scripted import ScriptedLM, scripted_tokenizer


def _eng(m, tok):
    return EngineV2(m, tok, EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2), max_model_len=256,
                                         use_cuda_graphs=False), eos_token_ids=[tok.eos_token_id])


def test_scripted_text_and_stop_strings():
    tok = scripted_tokenizer()
    prompt = tok.encode("Q: hi")
    m = ScriptedLM.from_text("Hello world. Bye", len(prompt), tok)
    eng = _eng(m, tok)
    s = eng.submit(Request(prompt_tokens=prompt, max_tokens=64, sampling=SamplingParams(temperature=0.0)))
    text = "".join(ev.text for ev in s)
    assert text == "Hello world. Bye"
    s2 = eng.submit(Request(prompt_tokens=prompt, max_tokens=64, sampling=SamplingParams(temperature=0.0),
                            stop_strings=["."]))
    assert "".join(ev.text for ev in s2) == "Hello world"


def test_scripted_tool_call_parsing():
    from mlx_swift_lm_b200.api.parsers import make_tool_parser

    tok = scripted_tokenizer()
    prompt = tok.encode("call")
    body = '<tool_call>{"name": "get_weather", "arguments": {"city": "Paris"}}</tool_call>'
    m = ScriptedLM.from_text(body, len(prompt), tok)
    eng = _eng(m, tok)
    s = eng.submit(Request(prompt_tokens=prompt, max_tokens=200, sampling=SamplingParams(temperature=0.0)))
    text = "".join(ev.text for ev in s)
    calls = make_tool_parser("hermes").parse(text)[1]
    assert calls and calls[0].name == "get_weather" and calls[0].arguments["city"] == "Paris"
