"""The reference-facing ten-function ABI (include/rpg_engine.h) end to end.

What an existing ctypes or Unity host does, on a synthetic model: load with a
config, read the model info, create a session, send chat requests (ChatML
rendering, tokenisation, prefill with reuse of the cached prompt prefix,
generate, detokenise, parse), reset the session, unload.  Mirrors the
reference's tests/abi_smoke.py checks: JSON shapes, finish reasons, usage
counts, deterministic greedy replies, errors on invalid handles.
"""

import ctypes
import json

import pytest

from rpgbarenginecuda_b200 import library_path

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    L = ctypes.CDLL(library_path())
    L.rpg_engine_load_model.restype = ctypes.c_int32
    L.rpg_engine_load_model.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
    L.rpg_engine_session_create.restype = ctypes.c_int32
    L.rpg_engine_session_create.argtypes = [ctypes.c_int32, ctypes.c_char_p]
    L.rpg_engine_generate.restype = ctypes.c_void_p
    L.rpg_engine_generate.argtypes = [ctypes.c_int32, ctypes.c_char_p]
    L.rpg_engine_model_info.restype = ctypes.c_void_p
    L.rpg_engine_model_info.argtypes = [ctypes.c_int32]
    L.rpg_engine_free.argtypes = [ctypes.c_void_p]
    L.rpg_engine_session_reset.restype = ctypes.c_int32
    L.rpg_engine_session_reset.argtypes = [ctypes.c_int32]
    L.rpg_engine_session_destroy.argtypes = [ctypes.c_int32]
    L.rpg_engine_unload_model.argtypes = [ctypes.c_int32]
    L.rpg_engine_last_error.restype = ctypes.c_char_p
    return L


def take_json(L, ptr, exact=None):
    """The reply as JSON; exact (a list) receives whether its bytes were valid
    UTF-8, i.e. whether its text round-trips to the same tokens."""
    assert ptr, L.rpg_engine_last_error().decode()
    try:
        raw = ctypes.string_at(ptr)
        if exact is not None:
            try:
                raw.decode("utf-8")
                exact.append(True)
            except UnicodeDecodeError:
                exact.append(False)
        # replies of a random-weight model may hold bytes that are not UTF-8
        return json.loads(raw.decode(errors="replace"))
    finally:
        L.rpg_engine_free(ptr)


def test_chat_round_trip(lib, tiny_model):
    L = lib
    m = L.rpg_engine_load_model(tiny_model.encode(), json.dumps({"context": 512, "device": 0}).encode())
    assert m >= 0, L.rpg_engine_last_error().decode()
    info = take_json(L, L.rpg_engine_model_info(m))
    assert info["n_layers"] == 2 and info["vocab"] == 4096
    s = L.rpg_engine_session_create(m, json.dumps({"max_seq": 512, "max_tokens": 8, "temperature": 0.0,
                                                   "seed": 1}).encode())
    assert s >= 0, L.rpg_engine_last_error().decode()
    req = {"messages": [{"role": "system", "content": "You are a shopkeeper."},
                        {"role": "user", "content": "What do you sell?"}],
           "max_tokens": 8, "temperature": 0.0}
    exact = []
    r1 = take_json(L, L.rpg_engine_generate(s, json.dumps(req).encode()), exact)
    assert isinstance(r1["text"], str)
    assert r1["finish_reason"] in ("stop", "length")
    assert 1 <= r1["usage"]["completion_tokens"] <= 8 and r1["usage"]["prompt_tokens"] > 0
    # A second turn reuses the cached prompt prefix (src/engine.cc:468-500):
    # the session keeps the KV rows of the longest common prefix and prefills
    # only the rest.  The reply must equal a fresh session's reply to the same
    # messages.  The assistant message is the first reply's text when its bytes
    # round-trip (then the whole first turn, generated tokens included, is
    # reused), else a fixed text (then the cache is cut back to the rendered
    # first prompt and reused up to there).
    assistant = r1["text"] if exact[0] else "We sell potions and maps."
    req2 = dict(req, messages=req["messages"] + [{"role": "assistant", "content": assistant},
                                                  {"role": "user", "content": "And the price?"}])
    r2 = take_json(L, L.rpg_engine_generate(s, json.dumps(req2).encode()))
    assert r2["usage"]["prompt_tokens"] > r1["usage"]["prompt_tokens"]
    fresh = L.rpg_engine_session_create(m, json.dumps({"max_seq": 512, "max_tokens": 8, "temperature": 0.0,
                                                       "seed": 1}).encode())
    assert fresh >= 0, L.rpg_engine_last_error().decode()
    r2f = take_json(L, L.rpg_engine_generate(fresh, json.dumps(req2).encode()))
    assert r2["text"] == r2f["text"] and r2["usage"] == r2f["usage"], (r2, r2f)
    L.rpg_engine_session_destroy(fresh)
    # greedy replies are deterministic: after a reset the first turn repeats
    assert L.rpg_engine_session_reset(s) == 0
    r3 = take_json(L, L.rpg_engine_generate(s, json.dumps(req).encode()))
    assert r3["text"] == r1["text"] and r3["usage"] == r1["usage"]
    # invalid handles fail with a message, then the engine keeps working
    assert L.rpg_engine_generate(s + 1000, json.dumps(req).encode()) is None
    assert L.rpg_engine_last_error()
    L.rpg_engine_session_destroy(s)
    L.rpg_engine_unload_model(m)
