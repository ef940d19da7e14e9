"""The host text layer of rpg_engine_generate against the reference's own host
code, byte for byte (CPU only).

The engine's tokenizer, ChatML prompt and output parse (csrc/abi_generate.cc,
through the rpgb_text_* entries of include/rpg_b200.h) are compared with the
reference's src/tokenizer.cc, src/chat_template.cc and src/tool_parser.cc,
compiled from its sources into oracle/_ref/libref_text.so, on the synthetic
GGUF's tokenizer:
* Encode ids (src/tokenizer.cc:314) with and without special-token matching;
* Decode bytes (src/tokenizer.cc:353), specials kept (src/engine.cc:565);
* the prompt of a request (src/engine.cc:452-464: ParseMessages, ParseTools,
  RenderChatml with the generation prompt and enable_thinking);
* ParseModelOutput (src/tool_parser.cc:125-178) as the response uses it
  (src/engine.cc:566-595): text, tool calls with their arguments or null, and
  the two unterminated flags.
Token ids and strings are byte work, so every comparison is exact.
"""

import json
import os

import numpy as np
import pytest

from oracle.oracle import REF_TEXT_SO
from rpgbarenginecuda_b200 import TextLayer, synthetic

pytestmark = pytest.mark.skipif(not os.path.exists(REF_TEXT_SO), reason="oracle/_ref not built")

TEXTS = [
    "", "a", "Hello, world!", "Hello world.  Two  spaces,\tone tab\nnew line\r\nCRLF",
    "   leading spaces", "trailing spaces   ", "\n\n\n", " \n \n", "12345678901234567890", "3.14159 and 2,718",
    "don't I'm you're we've they'll he'd it's", "DON'T I'M", "x's 'quoted' \"double\"",
    "你好，世界！这是一个测试。", "こんにちは世界", "안녕하세요", "Привет, мир", "مرحبا بالعالم", "café naïve résumé",
    "emoji 🙂👍🏽🚀 mixed", "math ∑∫√∞ ≤ ≥", "tabs\t\tand nbsp em space",
    "<|im_start|>user\nhi there<|im_end|>\n<|im_start|>assistant\n", "<think>\nreasoning\n</think>\n\nanswer",
    "<tool_call>\n{\"name\": \"f\", \"arguments\": {\"a\": 1}}\n</tool_call>", "<|im_start|><|im_end|><|endoftext|>",
    "<|im_start", "im_end|>", "<thinking>", "a<|im_end|>b<|im_end|>c",
    "code: def f(x):\n    return x**2  # comment\n", "URL https://example.com/path?q=1&r=2#frag",
    "$$$ ### @@@ !!! ??? ...", "MixedCASEwordsAndNumbers123abc456",
]

INVALID_UTF8 = [b"\xff\xfe", b"abc\x80def", b"\xc3", b"\xe4\xbd", b"ok\xf0\x9f\x99", b"\xed\xa0\x80", b"\x00mid\x00"]


@pytest.fixture(scope="module", params=["tiny", "qwen3-0.6b"])
def layers(request):
    from oracle.oracle import RefText

    path = synthetic.cached_model(request.param, seed=1 if request.param == "tiny" else 0)
    ours, ref = TextLayer(path), RefText(path)
    yield ours, ref
    ours.close()
    ref.close()


def random_texts(n, seed):
    rng = np.random.default_rng(seed)
    pieces = ["the", " quick", " brown", "fox", " 42", "\n", "  ", "\t", "é", "中文", "🙂", "'s", "'ll", ",", ".",
              "?!", "ab", "ba", "x", "123", " ", "Ü", "ß", "<think>", "<|im_end|>", "<tool_call>", "ẞ", "ǅ", "٣"]
    out = []
    for _ in range(n):
        k = int(rng.integers(1, 24))
        out.append("".join(pieces[int(i)] for i in rng.integers(0, len(pieces), size=k)))
    return out


@pytest.mark.parametrize("parse_special", [True, False])
def test_encode_ids_match_reference(layers, parse_special):
    ours, ref = layers
    for t in TEXTS + random_texts(300, 7):
        b = t.encode()
        assert ours.encode(b, parse_special) == ref.encode(b, parse_special), t


def test_encode_invalid_utf8_matches_reference(layers):
    ours, ref = layers
    for b in INVALID_UTF8:
        assert ours.encode(b, True) == ref.encode(b, True), b


def test_decode_bytes_match_reference(layers):
    ours, ref = layers
    rng = np.random.default_rng(3)
    vocab = 4096
    seqs = [ref.encode(t.encode()) for t in TEXTS]
    seqs += [list(rng.integers(0, vocab, size=int(rng.integers(1, 40)))) for _ in range(200)]
    seqs += [[], [vocab - 1], list(range(0, 300))]
    for ids in seqs:
        assert ours.decode(ids) == ref.decode(ids, skip_special=False), ids


def test_round_trip(layers):
    ours, _ = layers
    for t in TEXTS + random_texts(100, 9):
        assert ours.decode(ours.encode(t.encode())) == t.encode()


TOOLS = [
    {"type": "function", "function": {"name": "get_weather", "description": "Weather of a city",
                                      "parameters": {"type": "object", "properties": {"city": {"type": "string"}},
                                                     "required": ["city"]}}},
    {"type": "function", "function": {"name": "roll_dice", "description": "Rolls n dice",
                                      "parameters": {"type": "object", "properties": {"n": {"type": "integer"}}}}},
]

REQUESTS = [
    {"messages": [{"role": "user", "content": "Hello"}]},
    {"messages": [{"role": "system", "content": "You are a tavern keeper."}, {"role": "user", "content": "Ale!"}]},
    {"messages": [{"role": "user", "content": "Hi"}], "enable_thinking": False},
    {"messages": [{"role": "system", "content": "Sys"}, {"role": "user", "content": "q1"},
                  {"role": "assistant", "content": "a1"}, {"role": "user", "content": "q2"}]},
    {"messages": [{"role": "user", "content": "q1"},
                  {"role": "assistant", "content": "<think>\nstep one\nstep two\n</think>\n\nfinal a1"},
                  {"role": "user", "content": "q2"}]},
    {"messages": [{"role": "user", "content": "q1"},
                  {"role": "assistant", "content": "visible", "reasoning_content": "hidden thoughts"},
                  {"role": "user", "content": "q2"},
                  {"role": "assistant", "content": "last", "reasoning_content": "kept: after the last query"}]},
    {"messages": [{"role": "system", "content": "Use tools."}, {"role": "user", "content": "Weather in Oslo?"}],
     "tools": TOOLS},
    {"messages": [{"role": "user", "content": "Weather in Oslo?"}], "tools": TOOLS},
    {"messages": [{"role": "user", "content": "Weather?"}], "tools": []},
    {"messages": [{"role": "user", "content": "Weather in Oslo and Rome?"},
                  {"role": "assistant", "content": "",
                   "tool_calls": [{"type": "function", "function": {"name": "get_weather",
                                                                    "arguments": {"city": "Oslo"}}},
                                  {"type": "function", "function": {"name": "get_weather",
                                                                    "arguments": "{\"city\": \"Rome\"}"}}]},
                  {"role": "tool", "content": "{\"temp\": 3}"}, {"role": "tool", "content": "{\"temp\": 18}"},
                  {"role": "user", "content": "Thanks"}], "tools": TOOLS},
    {"messages": [{"role": "user", "content": "Roll"},
                  {"role": "assistant", "content": "Rolling now.",
                   "tool_calls": [{"name": "roll_dice", "arguments": {"n": 2, "sides": [1, 2.5, None, True]}}]},
                  {"role": "tool", "content": "7"}], "tools": TOOLS},
    {"messages": [{"role": "user", "content": "<tool_response>\nnot a real one\n</tool_response>"},
                  {"role": "assistant", "content": "ok"}]},
    {"messages": [{"role": "user", "content": "你好 🙂 café"}, {"role": "assistant", "content": "こんにちは"},
                  {"role": "user", "content": "Привет\n\n\ttab"}]},
    {"messages": [{"role": "system", "content": "first"}, {"role": "user", "content": "u"},
                  {"role": "system", "content": "second system"}, {"role": "user", "content": "v"}]},
    {"messages": [{"role": "assistant", "content": "<think>unclosed reasoning"}, {"role": "user", "content": "u"}]},
    {"messages": [{"role": "user", "content": "u"},
                  {"role": "assistant", "content": "<think>\n</think>\n\nempty thought"}]},
    {"messages": [{"role": "user", "content": "a \"quoted\" \\ backslash / slash \u0001 control"}],
     "tools": [{"type": "function", "function": {"name": "w", "description": "unicode é 中 🙂 \"q\" \\"}}]},
]


@pytest.mark.parametrize("i", range(len(REQUESTS)))
def test_rendered_prompt_matches_reference(layers, i):
    ours, ref = layers
    req = REQUESTS[i]
    tools = json.dumps(req["tools"]) if "tools" in req else None
    want = ref.render(json.dumps(req["messages"]), tools, True, req.get("enable_thinking", True))
    got = ours.render(json.dumps(req))
    assert got == want
    # and the ids the engine prefills
    assert ours.encode(got, True) == ref.encode(want, True)


OUTPUTS = [
    "Plain answer.", "  padded answer \n\n", "<think>\nreasoning here\n</think>\n\nThe answer is 4.",
    "<think>never closed reasoning", "before<think>mid</think>after", "<think>a</think>x<think>b</think>y",
    "<tool_call>\n{\"name\": \"get_weather\", \"arguments\": {\"city\": \"Oslo\"}}\n</tool_call>",
    "Sure.<tool_call>\n{\"name\": \"roll_dice\", \"arguments\": \"{\\\"n\\\": 3}\"}\n</tool_call>",
    "<tool_call>{\"name\": \"a\", \"arguments\": {}}</tool_call><tool_call>{\"name\": \"b\", \"arguments\": "
    "{\"x\": [1, 2]}}</tool_call>",
    "<tool_call>\n{\"name\": \"bad\", \"arguments\": [1, 2]}\n</tool_call>",
    "<tool_call>\nnot json at all\n</tool_call>", "<tool_call>\n{\"name\": \"cut\", \"argum",
    "<tool_call>{\"arguments\": {\"a\": 1}}</tool_call>",
    "text<|im_end|>", "<|im_start|>assistant\nhello<|im_end|><|endoftext|>", "<|im_start|>user\nq<|im_end|>",
    "<|im_start|>weird\nx", "<think>\n\n</think>\n\n<tool_call>\n{\"name\": \"f\", \"arguments\": {\"k\": "
    "\"v é 中\"}}\n</tool_call>\ntrailing text",
    "unicode 中文 🙂 é", "", "<tool_call></tool_call>", "<tool_call>{\"name\": \"n\", \"arguments\": \"not an object\"}"
    "</tool_call>",
]


@pytest.mark.parametrize("i", range(len(OUTPUTS)))
def test_output_parse_matches_reference(layers, i):
    ours, ref = layers
    raw = OUTPUTS[i].encode()
    got = json.loads(ours.parse(raw))
    want = json.loads(ref.parse(raw))
    assert got["text"] == want["text"]
    assert got["unterminated_think"] == want["unterminated_think"]
    assert got["unterminated_tool_call"] == want["unterminated_tool_call"]
    assert len(got["tool_calls"]) == len(want["tool_calls"])
    for g, w in zip(got["tool_calls"], want["tool_calls"]):
        assert g["name"] == w["name"]
        assert g["arguments"] == (json.loads(w["arguments"]) if w["ok"] else None)
