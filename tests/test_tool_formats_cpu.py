"""Tool-call formats: each family's syntax parses to the same call, whole and
streamed one character at a time (frames split anywhere), with the text
around frames kept as content and schema-typed argument values."""
import pytest

from mlx_swift_lm_b200.api.parsers import make_tool_parser
from mlx_swift_lm_b200.api.tool_formats import infer_tool_format

TOOLS = [{"type": "function", "function": {"name": "get_weather", "parameters": {
    "type": "object", "properties": {"city": {"type": "string"}, "days": {"type": "integer"},
                                     "units": {"type": ["string", "null"]}, "tags": {"type": "array"}},
    "required": ["city"]}}}]
WANT = {"city": "Tokyo", "days": 3}

CASES = {
    "json": '<tool_call>{"name": "get_weather", "arguments": {"city": "Tokyo", "days": 3}}</tool_call>',
    "hermes": '<tool_call>\n{"name": "get_weather", "arguments": {"city": "Tokyo", "days": 3}}\n</tool_call>',
    "xml_function": "<tool_call>\n<function=get_weather>\n<parameter=city>\nTokyo\n</parameter>\n"
                    "<parameter=days>\n3\n</parameter>\n</function>\n</tool_call>",
    "nemotron": "<function=get_weather><parameter=city>Tokyo</parameter><parameter=days>3</parameter></function>",
    "qwen3_5": "<tool_call>\n<function=get_weather>\n<parameter=city>\nTokyo\n</parameter>\n<parameter=days>\n3\n"
               "</parameter>\n</function>\n</tool_call>",
    "mimo_v2": "<tool_call><function=get_weather><parameter=city>Tokyo</parameter><parameter=days>3</parameter>"
               "</function></tool_call>",
    "glm4": "<tool_call>get_weather\n<arg_key>city</arg_key>\n<arg_value>Tokyo</arg_value>\n<arg_key>days</arg_key>\n"
            "<arg_value>3</arg_value>\n</tool_call>",
    "glm5": "<tool_call>get_weather<arg_key>city</arg_key><arg_value>Tokyo</arg_value><arg_key>days</arg_key>"
            "<arg_value>3</arg_value></tool_call>",
    "flint": "<tool_call>get_weather<arg_key>city</arg_key><arg_value>Tokyo</arg_value><arg_key>days</arg_key>"
             "<arg_value>3</arg_value></tool_call>",
    "gemma4": '<|tool_call>call:get_weather{city:<|"|>Tokyo<|"|>,days:3}<tool_call|>',
    "gemma": "<start_function_call>call:get_weather{city:<escape>Tokyo<escape>,days:3}<end_function_call>",
    "kimi_k2": "<|tool_calls_section_begin|><|tool_call_begin|>functions.get_weather:0<|tool_call_argument_begin|>"
               '{"city": "Tokyo", "days": 3}<|tool_call_end|><|tool_calls_section_end|>',
    "minimax_m2": '<minimax:tool_call>\n<invoke name="get_weather">\n<parameter name="city">Tokyo</parameter>\n'
                  '<parameter name="days">3</parameter>\n</invoke>\n</minimax:tool_call>',
    "atem": '<atem:function_calls><atem:invoke name="get_weather"><atem:parameter name="city">Tokyo'
            '</atem:parameter><atem:parameter name="days">3</atem:parameter></atem:invoke></atem:function_calls>',
    "mistral": '[TOOL_CALLS]get_weather[ARGS]{"city": "Tokyo", "days": 3}',
    "llama3": '<|python_tag|>{"name": "get_weather", "parameters": {"city": "Tokyo", "days": 3}}',
    "lfm2": "<|tool_call_start|>[get_weather(city='Tokyo', days=3)]<|tool_call_end|>",
}


@pytest.mark.parametrize("fmt", sorted(CASES))
def test_format_whole_and_streamed(fmt):
    text = "Let me check. " + CASES[fmt]
    content, calls = make_tool_parser(fmt, TOOLS).parse(text)
    assert [c.name for c in calls] == ["get_weather"], (fmt, calls)
    assert calls[0].arguments == WANT
    assert content.strip() == "Let me check."
    p = make_tool_parser(fmt, TOOLS)
    got_c, got_calls = [], []
    for ch in text:
        c, cs = p.feed(ch)
        got_c.append(c)
        got_calls += cs
    c, cs = p.flush()
    got_c.append(c)
    got_calls += cs
    assert [(c.name, c.arguments) for c in got_calls] == [("get_weather", WANT)], fmt
    assert "".join(got_c).strip() == "Let me check."
    # no frame text leaks into streamed content
    assert "<" not in "".join(got_c) and "[TOOL" not in "".join(got_c)


def test_string_typed_values_stay_raw():
    # a declared string that looks like JSON stays text; an undeclared value parses
    txt = "<tool_call><function=get_weather><parameter=city>123</parameter><parameter=extra>[1, 2]</parameter>" \
          "</function></tool_call>"
    _, calls = make_tool_parser("xml_function", TOOLS).parse(txt)
    assert calls[0].arguments == {"city": "123", "extra": [1, 2]}


def test_qwen35_json_dialect_and_multiple_calls():
    txt = ('<tool_call>{"name": "get_weather", "arguments": {"city": "Oslo"}}</tool_call>\n'
           "<tool_call><function=get_weather><parameter=city>Rome</parameter></function></tool_call>")
    _, calls = make_tool_parser("qwen3_5", TOOLS).parse(txt)
    assert [c.arguments["city"] for c in calls] == ["Oslo", "Rome"]


def test_mistral_call_id_and_legacy_list():
    _, calls = make_tool_parser("mistral").parse('[TOOL_CALLS]get_weather[CALL_ID]abc123[ARGS]{"city": "Paris"}')
    assert calls[0].id == "abc123" and calls[0].arguments == {"city": "Paris"}
    _, calls = make_tool_parser("mistral").parse('[TOOL_CALLS][{"name": "a", "arguments": {}}, '
                                                 '{"name": "b", "arguments": {"x": 1}}]')
    assert [c.name for c in calls] == ["a", "b"]


def test_gemma_nested_values_and_lists():
    txt = '<|tool_call>call:f{a:{b:<|"|>x, y<|"|>,c:[1,2,true]},d:null}<tool_call|>'
    _, calls = make_tool_parser("gemma4").parse(txt)
    assert calls[0].arguments == {"a": {"b": "x, y", "c": [1, 2, True]}, "d": None}


def test_pythonic_multiple_calls():
    _, calls = make_tool_parser("lfm2").parse("<|tool_call_start|>[f(a='x', b=[1, 2]), g()]<|tool_call_end|>")
    assert [(c.name, c.arguments) for c in calls] == [("f", {"a": "x", "b": [1, 2]}), ("g", {})]


def test_glm4_markerless_named_json_only_for_declared_tools():
    _, calls = make_tool_parser("glm4", TOOLS).parse('<tool_call>get_weather\n{"city": "Lima"}</tool_call>')
    assert calls[0].arguments == {"city": "Lima"}
    _, calls = make_tool_parser("glm4", TOOLS).parse('<tool_call>unknown_tool\n{"city": "Lima"}</tool_call>')
    assert calls == []


def test_json_bare_recovery_and_unterminated_frame():
    _, calls = make_tool_parser("json").parse('{"name": "get_weather", "arguments": {"city": "Kyiv"}}')
    assert calls[0].arguments == {"city": "Kyiv"}
    # end-of-sequence inside a frame: the frame is parsed as if closed
    p = make_tool_parser("json")
    c, cs = p.feed('ok <tool_call>{"name": "f", "arguments": {}}')
    c2, cs2 = p.flush()
    assert (c + c2).strip() == "ok" and [x.name for x in cs + cs2] == ["f"]


def test_format_inference():
    assert infer_tool_format("qwen3_5_moe") == "qwen3_5"
    assert infer_tool_format("gemma4_text") == "gemma4"
    assert infer_tool_format("gpt_oss") == "harmony"
    assert infer_tool_format("unknown") == "json"
